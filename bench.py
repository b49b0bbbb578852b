#!/usr/bin/env python
"""Benchmark of the det decode path at the Gemma-4-E4B (stand-in) shape.

One step = one greedy token of the reference's decode loop
(executors/native.rs:265-450): select_output_token (argmax_first over the
logits) followed by decode_transition (embedding, PLE input, every layer with
its KV append and attention over the 4096-token context, final norm,
lm_head, softcap).  The model is the seeded random-init E4B stand-in
(raster-inference_b200/configs/e4b_text_standin.json, i16 weights, ~15 GB in
HBM); the prompt is 4096 seeded uniform-random token ids, prefilled on the GPU
before timing.  Each step streams every weight once (~9 GB > L2), so no L2
flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Multi-GPU: the decode of one sequence is not sharded here; each rank runs an
independent replica (its own sequence), timed on the device and reduced with
the max over ranks ("scaling": "weak").

Also reported: the det-GEMV roofline (E4B projection shapes, CUDA events on
the launching stream), prefill tok/s of the 4096-token prompt, the end-to-end
number through the C ABI with host buffers, and the CPU baseline (the C++
restatement of the reference det path on the host cores, a bounded sample).
"""
import argparse
import hashlib
import importlib
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
METRIC = "det decode & prefill tok/s (E4B shape, bit-exact); det-GEMV HBM GB/s vs peak"
CONFIG_PATH = os.path.join(ROOT, "raster-inference_b200", "configs", "e4b_text_standin.json")
SEED = 20260501


def lcg_ids(n, vocab, seed):
    s, out = seed, []
    for _ in range(n):
        s = (s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        out.append((s >> 33) % vocab)
    return out


def load_fixtures():
    """The CPU oracle's E4B-shape results (tests/golden/e4b_fixtures.json), or None."""
    path = os.path.join(ROOT, "tests", "golden", "e4b_fixtures.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f)


def load_config():
    with open(CONFIG_PATH) as f:
        return json.load(f)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.p:
            self.p.terminate()
            try:
                out, _ = self.p.communicate(timeout=10)
            except Exception:
                self.p.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm),
                "window": "from the 4096-token prefills through the timed decode steps"}


# ---------------------------------------------------------------------------
# CPU: the oracle (C++ restatement of the reference det path) on host cores
# ---------------------------------------------------------------------------
def cpu_decode_rate(cfg, ctx, steps, threads, single_thread_steps=0):
    """Greedy decode steps of the CPU oracle at context ctx (seeded synthetic
    KV cache) on `threads` host threads, then `single_thread_steps` more on
    one thread.  Returns (times, single-thread times, setup seconds)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O  # CPU baseline only
    O.set_threads(threads)
    t0 = time.perf_counter()
    m = O.Model(None, synthetic=(cfg, SEED, 16))
    s = m.seq()
    s.fill_synthetic(ctx, seed=7)
    setup = time.perf_counter() - t0
    tok = 1

    def run(n):
        nonlocal tok
        out = []
        for _ in range(n):
            t = time.perf_counter()
            _, logits, _ = s.decode(tok, want_layer_hashes=False)
            tok = O.argmax_first(logits)
            out.append(time.perf_counter() - t)
        return out

    times = run(steps)
    single = []
    if single_thread_steps:
        O.set_threads(1)
        single = run(single_thread_steps)
        O.set_threads(threads)
    m.close()
    return times, single, setup


def config1_routines(rdet):
    """the reference's tiny-gemma-dev bundle, a 16-token
    prompt (LCG seed 0 over its 280-token vocabulary), prefill and 8 greedy
    tokens, wall time per routine through the C ABI (host-synchronous calls)
    and through the CPU oracle, tokens and commitments compared."""
    import tempfile
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import tiny_gemma_dev  # fixture writer: regenerates the reference's bundle bytes
    import oracle as O  # checker and CPU timing only
    detwgt = importlib.import_module("raster-inference_b200.detwgt")
    d = tiny_gemma_dev.write_bundle(tempfile.mkdtemp(prefix="rdet-c1-"), detwgt.encode)
    ids = tiny_gemma_dev.lcg_token_ids(16, 280, 0)
    out = {"prompt_tokens": 16, "new_tokens": 8}
    m = rdet.Model.open(d, max_prefill=16)
    res = {}
    for rep in range(2):  # the first pass warms up
        t = {"input.embedding": 0.0, "prefill": 0.0, "select_output_token": 0.0, "decode_transition": 0.0}
        s = m.new_sequence(32)
        c0 = time.perf_counter()
        m.embed(ids)
        t["input.embedding"] = time.perf_counter() - c0
        c0 = time.perf_counter()
        s.prefill(ids)
        t["prefill"] = time.perf_counter() - c0
        toks = []
        for _ in range(8):
            c0 = time.perf_counter()
            tok = s.select()
            t["select_output_token"] += (time.perf_counter() - c0) / 8
            toks.append(tok)
            c0 = time.perf_counter()
            s.decode(tok)
            t["decode_transition"] += (time.perf_counter() - c0) / 8
        res = {"ms": {k: round(1000 * v, 4) for k, v in t.items()}, "tokens": toks,
               "kv": s.commitment(rdet.BUF_KV), "logits": s.commitment(rdet.BUF_LOGITS)}
        s.free()
    m.close()
    om = O.Model(d, threads=1)
    t = {"input.embedding": 0.0, "prefill": 0.0, "select_output_token": 0.0, "decode_transition": 0.0}
    os_ = om.seq()
    c0 = time.perf_counter()
    om.embed(ids)
    t["input.embedding"] = time.perf_counter() - c0
    c0 = time.perf_counter()
    _, logits, _ = os_.prefill(ids, want_layer_hashes=False)
    t["prefill"] = time.perf_counter() - c0
    ctoks = []
    for _ in range(8):
        c0 = time.perf_counter()
        tok = O.argmax_first(logits)
        t["select_output_token"] += (time.perf_counter() - c0) / 8
        ctoks.append(tok)
        c0 = time.perf_counter()
        _, logits, _ = os_.decode(tok, want_layer_hashes=False)
        t["decode_transition"] += (time.perf_counter() - c0) / 8
    out["gpu_ms_per_routine"] = res["ms"]
    out["cpu_ms_per_routine"] = {k: round(1000 * v, 4) for k, v in t.items()}
    out["cpu_threads"] = 1
    out["bit_exact_vs_cpu"] = (res["tokens"] == ctoks and res["kv"] == os_.kv_commitment() and
                               res["logits"] == O.vec_commitment(logits))
    out["tokens"] = res["tokens"]
    om.close()
    return out


def run_reference(args, rank):
    if rank != 0:
        return  # the CPU arm runs on rank 0 only
    cfg = load_config()
    cores = host_cores()
    times, _, _ = cpu_decode_rate(cfg, args.ctx, args.warmup + args.steps, cores)
    timed = times[args.warmup:]
    total = sum(timed)
    value = len(timed) / total
    sample = (f"{len(timed)} greedy decode steps at context {args.ctx} (seeded synthetic KV cache) on the E4B stand-in, "
              f"{cores} threads, {cpu_model()}")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / len(timed),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int64",
            "data": "synthetic (seeded random-init weights of the E4B stand-in shape)",
            "config": {"workload": "det greedy decode, batch 1, context 4096, E4B stand-in (config 4)",
                       "model": "gemma-4-e4b-text-standin", "context": args.ctx},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores,
                             "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def e4b_gemv_shapes(cfg):
    t = cfg["text_config"]
    H, F, Hq, kv, d, dg, V, P, L = (t["hidden_size"], t["intermediate_size"], t["num_attention_heads"],
                                    t["num_key_value_heads"], t["head_dim"], t["global_head_dim"],
                                    t["vocab_size"], t["hidden_size_per_layer_input"], t["num_hidden_layers"])
    return {"q": (Hq * d, H), "k": (kv * d, H), "v": (kv * d, H), "o": (H, Hq * d), "gate": (F, H),
            "up": (F, H), "down": (H, F), "q_full": (Hq * dg, H), "o_full": (H, Hq * dg),
            "ple_model_proj": (L * P, H), "lm_head": (V, H)}


def decode_step_bytes(cfg, ctx):
    """Algorithmic HBM bytes of one decode step at context ctx: every weight a
    decode GEMV streams (i16; the KV-sharing layers' unused k/v projections
    excluded), the KV rows each layer's attention reads and the rows it
    appends, the PLE model projection and lm_head."""
    t = cfg["text_config"]
    H, F, Hq, kv, d, dg, V, P, L, W = (t["hidden_size"], t["intermediate_size"], t["num_attention_heads"],
                                       t["num_key_value_heads"], t["head_dim"], t["global_head_dim"],
                                       t["vocab_size"], t["hidden_size_per_layer_input"], t["num_hidden_layers"],
                                       t["sliding_window"])
    shared = t.get("num_kv_shared_layers") or 0
    total = L * P * H * 2 + V * H * 2
    for l, lt in enumerate(t["layer_types"]):
        sliding = lt == "sliding_attention"
        hd = d if sliding else dg
        rows = min(ctx, W) if sliding else ctx
        total += (Hq * hd * H + H * Hq * hd + 3 * F * H + 2 * P * H) * 2
        total += 2 * kv * hd * rows * 4
        if l < L - shared:
            total += 2 * kv * hd * H * 2 + 2 * kv * hd * 4
    return total


INT8_PEAK_OPS = 4.5e15  # B200 dense int8 tensor ops/s, nominal (no measured int8 figure on this pool)


def prefill_int8_ops(cfg, S):
    """int8 tensor-core ops (2 per multiply-add) of one S-token prefill:
    every projection as 8 byte-limb products per det multiply-add (4
    activation limbs x 2 weight limbs of i16 weights; the KV-sharing layers'
    unused k/v projections excluded), the PLE model projection, and the
    attention's 16 (scores) + 12 (weighted values) limb products per (query,
    key, dim) of each head.  lm_head runs as a GEMV on the last row only."""
    t = cfg["text_config"]
    H, F, Hq, kv, d, dg, P, L, W = (t["hidden_size"], t["intermediate_size"], t["num_attention_heads"],
                                    t["num_key_value_heads"], t["head_dim"], t["global_head_dim"],
                                    t["hidden_size_per_layer_input"], t["num_hidden_layers"], t["sliding_window"])
    shared = t.get("num_kv_shared_layers") or 0
    macs = L * P * H * S * 8
    for l, lt in enumerate(t["layer_types"]):
        sliding = lt == "sliding_attention"
        hd = d if sliding else dg
        proj = Hq * hd * H + H * Hq * hd + 3 * F * H + 2 * P * H + (2 * kv * hd * H if l < L - shared else 0)
        macs += proj * S * 8
        pairs = sum(min(i + 1, W) for i in range(S)) if sliding else S * (S + 1) // 2
        macs += Hq * hd * pairs * 28
    return 2 * macs


def gemv_roofline(torch, rdet, cfg, device, copies=8, rounds=3, check=False):
    """det-GEMV (gemv3_kernel) at the E4B projection shapes.  For each shape,
    `copies` launches over distinct weight copies run back to back on one
    stream (as inside the decode step) between two CUDA events on that
    stream; the mean per launch is the launch duration.  Between two uses of
    one copy every other shape streams (> L2), so each launch reads HBM."""
    shapes = e4b_gemv_shapes(cfg)
    g = torch.Generator(device=f"cuda:{device}").manual_seed(3)
    dev = f"cuda:{device}"
    mats = {k: [torch.randint(-32768, 32768, s, dtype=torch.int16, device=dev, generator=g)
                for _ in range(copies if k != "lm_head" else 2)] for k, s in shapes.items()}
    # activations: N(0, 1) quantized with f32_to_act
    detwgt = importlib.import_module("raster-inference_b200.detwgt")
    xs = {k: torch.from_numpy(detwgt.normal_acts(s[1], 1000 + n)).to(dev) for n, (k, s) in enumerate(shapes.items())}
    ys = {k: torch.empty(s[0], dtype=torch.int32, device=dev) for k, s in shapes.items()}
    stream = torch.cuda.Stream(device=device)
    per = {k: [] for k in shapes}
    with torch.cuda.stream(stream):
        for r in range(rounds + 1):
            for k, (n, kk) in shapes.items():
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for m in mats[k]:
                    rdet.det_gemv(xs[k].data_ptr(), m.data_ptr(), 16, n, kk, ys[k].data_ptr(), stream.cuda_stream)
                e1.record(stream)
                if r >= 1:
                    per[k].append((e0, e1, len(mats[k])))
    stream.synchronize()
    # bit check of every output row of the first weight copy against the CPU
    # det GEMV (outside the timed region)
    bit_exact = None
    if check:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O  # checker only
        bit_exact = True
        for k, (n, kk) in shapes.items():
            with torch.cuda.stream(stream):
                rdet.det_gemv(xs[k].data_ptr(), mats[k][0].data_ptr(), 16, n, kk, ys[k].data_ptr(),
                              stream.cuda_stream)
            stream.synchronize()
            if not (ys[k].cpu().numpy() == O.gemv(xs[k].cpu().numpy(), mats[k][0].cpu().numpy())).all():
                bit_exact = False
    out, tot_b, tot_t = {}, 0.0, 0.0
    for k, (n, kk) in shapes.items():
        ms = statistics.mean(a.elapsed_time(b) / c for a, b, c in per[k])
        b = n * kk * 2 + kk * 4 + n * 4
        out[k] = {"rows": n, "cols": kk, "us": ms * 1000, "gbs": b / (ms * 1e-3) / 1e9}
        tot_b += b
        tot_t += ms * 1e-3
    return out, tot_b / tot_t / 1e9, tot_b / len(shapes), tot_t / len(shapes), bit_exact


def run_kernel_case(args):
    """A few launches of one kernel at E4B shapes, sized for an ncu capture
    (a few GB on the device): --kernel-case gemv runs gemv3 on the q, down and
    lm_head shapes; --kernel-case attn runs the cluster decode attention of a
    sliding and a full layer at context --ctx."""
    import torch
    rdet = importlib.import_module("raster-inference_b200")
    cfg = load_config()
    t = cfg["text_config"]
    dev = "cuda:0"
    g = torch.Generator(device=dev).manual_seed(5)
    if args.kernel_case == "prefill":
        # one prefill of the --ctx-token prompt at E4B shape inside the NVTX
        # range "prefill" (after an unrecorded prefill that does first-use
        # setup), for a launch list filtered with --nvtx-include "prefill/"
        model = rdet.Model.synthetic(cfg, SEED, width=16, device=0, max_prefill=args.ctx)
        ids = lcg_ids(args.ctx, t["vocab_size"], SEED)
        for rep in range(2):
            seq = model.new_sequence(args.ctx + 8)
            torch.cuda.synchronize()
            if rep:
                torch.cuda.nvtx.range_push("prefill")
            seq.prefill(ids)
            torch.cuda.synchronize()
            if rep:
                torch.cuda.nvtx.range_pop()
            seq.free()
        model.close()
        print(f"prefill: {args.ctx} tokens")
        return
    if args.kernel_case == "batchattn":
        # the batched decode attention alone at config-5 lengths: a narrow
        # model with the E4B head geometry (sliding layer, full layer), 64
        # ragged sequences, three batched steps (a few GB on the device)
        small = {"text_config": dict(t, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                                     num_kv_shared_layers=1, vocab_size=300, vocab_size_per_layer_input=300,
                                     hidden_size_per_layer_input=32,
                                     layer_types=["sliding_attention", "full_attention", "sliding_attention",
                                                  "sliding_attention"])}
        model = rdet.Model.synthetic(small, SEED, width=16, device=0, max_prefill=args.ctx)
        lens = [128 + (x % 3969) for x in lcg_ids(args.batch, 1 << 30, SEED + 7)]
        seqs = [model.new_sequence(n + 16) for n in lens]
        for i, (sq, n) in enumerate(zip(seqs, lens)):
            sq.prefill(lcg_ids(n, 300, SEED + 100 + i))
        toks = rdet.select_batch(model, seqs)
        for rep in range(3):
            rdet.decode_batch(model, seqs, toks)
            toks = rdet.select_batch(model, seqs)
        model.close()
        print(f"batched decode attention: {args.batch} sequences, 3 steps")
        return
    if args.kernel_case == "batch":
        # one greedy step of the 64-sequence ragged batch
        # inside the NVTX range "batch", after two untimed steps, for a launch
        # list filtered with --nvtx-include "batch/"
        model = rdet.Model.synthetic(cfg, SEED, width=16, device=0, max_prefill=args.ctx)
        lens = [128 + (x % 3969) for x in lcg_ids(args.batch, 1 << 30, SEED + 7)]
        seqs = [model.new_sequence(n + 16) for n in lens]
        for i, (sq, n) in enumerate(zip(seqs, lens)):
            sq.prefill(lcg_ids(n, t["vocab_size"], SEED + 100 + i))
        toks = rdet.select_batch(model, seqs)
        for rep in range(3):
            torch.cuda.synchronize()
            if rep == 2:
                torch.cuda.nvtx.range_push("batch")
            rdet.decode_batch(model, seqs, toks)
            toks = rdet.select_batch(model, seqs)
            torch.cuda.synchronize()
            if rep == 2:
                torch.cuda.nvtx.range_pop()
        model.close()
        print(f"batched decode step: {args.batch} sequences")
        return
    if args.kernel_case == "convert":
        # model ingestion: a vocab x hidden bf16 tensor (lm_head-sized) to Q16.16
        # on the GPU (device time, CUDA events) and through convert.py's GPU
        # path with the host<->device copies, beside the host form
        convert = importlib.import_module("raster-inference_b200.convert")
        import numpy as np
        rows, cols = t["vocab_size"], t["hidden_size"]
        rng = np.random.default_rng(3)
        w = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
        raw = (w.view(np.uint32) >> 16).astype("<u2").tobytes()
        src = torch.from_numpy(np.frombuffer(raw, dtype=np.uint8).copy()).to(dev)
        out = torch.empty(rows * cols, dtype=torch.int32, device=dev)
        mass = torch.empty(rows, dtype=torch.int64, device=dev)
        stats = torch.zeros(2, dtype=torch.int32, device=dev)
        rdet.convert_to_wgt(src.data_ptr(), "BF16", rows, cols, out.data_ptr(), mass.data_ptr(), stats.data_ptr())
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        rdet.convert_to_wgt(src.data_ptr(), "BF16", rows, cols, out.data_ptr(), mass.data_ptr(), stats.data_ptr())
        e1.record()
        torch.cuda.synchronize()
        dev_s = e0.elapsed_time(e1) / 1000
        t0 = time.perf_counter()
        gb, gm = convert.convert_tensor_gpu(memoryview(raw), "BF16", (rows, cols), 0)
        gpu_s = time.perf_counter() - t0
        from concurrent.futures import ThreadPoolExecutor
        with ThreadPoolExecutor(max_workers=host_cores()) as pool:
            t0 = time.perf_counter()
            hb, hm = convert.convert_tensor(memoryview(raw), "BF16", (rows, cols), pool)
            host_s = time.perf_counter() - t0
        n = rows * cols
        print(json.dumps({"case": "convert bf16", "values": n, "device_gvalues_s": n / dev_s / 1e9,
                          "device_gbs": n * 6 / dev_s / 1e9, "gpu_path_gvalues_s": n / gpu_s / 1e9,
                          "host_gvalues_s": n / host_s / 1e9, "host_cores": host_cores(),
                          "identical": bool(np.array_equal(gb, hb) and np.array_equal(gm, hm))}))
        return
    if args.kernel_case == "tcattn":
        # prefill attention on the tensor cores (rdet_det_attention_prefill) for
        # a full layer (head_dim 512, causal) and a sliding layer (head_dim 256,
        # window 512) of a --ctx-token prompt at the E4B head counts
        Hq, kv, d, dg, win = (t["num_attention_heads"], t["num_key_value_heads"], t["head_dim"],
                              t["global_head_dim"], t["sliding_window"])
        S = args.ctx
        for name, hd, w in (("full", dg, 0), ("sliding", d, win)):
            q = torch.randint(-(1 << 18), 1 << 18, (S, Hq, hd), dtype=torch.int32, device=dev, generator=g)
            kc = torch.randint(-(1 << 18), 1 << 18, (kv, S, hd), dtype=torch.int32, device=dev, generator=g)
            vc = torch.randint(-(1 << 20), 1 << 20, (kv, S, hd), dtype=torch.int32, device=dev, generator=g)
            out = torch.empty((S, Hq, hd), dtype=torch.int32, device=dev)
            rdet.det_attention_prefill(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), S, S, Hq, kv, hd, w,
                                       out.data_ptr())
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            rdet.det_attention_prefill(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), S, S, Hq, kv, hd, w,
                                       out.data_ptr())
            e1.record()
            torch.cuda.synchronize()
            keys = sum(min(i + 1, w) if w else i + 1 for i in range(S))
            print(f"tc attn {name}: S {S} heads {Hq}/{kv} head_dim {hd} window {w} ms {e0.elapsed_time(e1):.3f} "
                  f"score MACs {Hq * hd * keys} int8 limb MACs {Hq * hd * keys * 28}")
        return
    if args.kernel_case == "tc":
        # prefill linear on the tensor cores (rdet_det_linear, >= 32 rows): byte-plane
        # prep kernels then tc_linear_kernel, at 2048 prompt tokens
        shapes = e4b_gemv_shapes(cfg)
        S = 2048
        for k in ("gate", "down", "q"):
            n, kk = shapes[k]
            w = torch.randint(-32768, 32768, (n, kk), dtype=torch.int16, device=dev, generator=g)
            x = torch.randint(-(1 << 20), 1 << 20, (S, kk), dtype=torch.int32, device=dev, generator=g)
            y = torch.empty((S, n), dtype=torch.int32, device=dev)
            rdet.det_linear(x.data_ptr(), S, w.data_ptr(), 16, n, kk, y.data_ptr())
            torch.cuda.synchronize()
            print(f"tc linear {k}: S {S} rows {n} cols {kk} int8 limb MACs {8 * S * n * kk}")
        return
    if args.kernel_case == "gemv":
        shapes = e4b_gemv_shapes(cfg)
        for k in ("q", "down", "lm_head"):
            n, kk = shapes[k]
            w = torch.randint(-32768, 32768, (n, kk), dtype=torch.int16, device=dev, generator=g)
            x = torch.randint(-(1 << 20), 1 << 20, (kk,), dtype=torch.int32, device=dev, generator=g)
            y = torch.empty(n, dtype=torch.int32, device=dev)
            rdet.det_gemv(x.data_ptr(), w.data_ptr(), 16, n, kk, y.data_ptr())
            torch.cuda.synchronize()
            print(f"gemv {k}: rows {n} cols {kk} bytes {n * kk * 2 + kk * 4 + n * 4}")
    else:
        Hq, kv, d, dg, win = (t["num_attention_heads"], t["num_key_value_heads"], t["head_dim"],
                              t["global_head_dim"], t["sliding_window"])
        ctx = args.ctx
        for name, hd, w in (("sliding", d, win), ("full", dg, 0)):
            cap = ctx + 64
            q = torch.randint(-(1 << 17), 1 << 17, (Hq, hd), dtype=torch.int32, device=dev, generator=g)
            kc = torch.randint(-(1 << 17), 1 << 17, (kv, cap, hd), dtype=torch.int32, device=dev, generator=g)
            vc = torch.randint(-(1 << 20), 1 << 20, (kv, cap, hd), dtype=torch.int32, device=dev, generator=g)
            out = torch.empty((Hq, hd), dtype=torch.int32, device=dev)
            pos = ctx - 1
            rdet.det_attention_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), cap, Hq, kv, hd, pos, w,
                                      out.data_ptr())
            torch.cuda.synchronize()
            rows = min(pos + 1, w) if w else pos + 1
            line = f"attn {name}: heads {Hq}/{kv} head_dim {hd} rows {rows} kv_bytes {2 * kv * rows * hd * 4}"
            if args.time_calls:
                # per-call time of the allocating entry point (cluster kernel)
                # and of the allocation-free one (split-phase kernels), CUDA
                # events around back-to-back calls on the default stream
                us = {}
                for label, fn in (("alloc", rdet.det_attention_decode),
                                  ("noalloc", rdet.det_attention_decode_noalloc)):
                    fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), cap, Hq, kv, hd, pos, w, out.data_ptr())
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    for _ in range(args.time_calls):
                        fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), cap, Hq, kv, hd, pos, w, out.data_ptr())
                    e1.record()
                    torch.cuda.synchronize()
                    us[label] = 1000 * e0.elapsed_time(e1) / args.time_calls
                line += f" us_per_call alloc {us['alloc']:.1f} noalloc {us['noalloc']:.1f}"
            print(line)


def batched_run(args, torch, rdet, dist, model, stream, t, rank, world, local_rank, mode):
    """64 sequences, prompt lengths 128 + draw % 3969
    (seeded), greedy: one batched decode_transition per step, then
    select_output_token for every sequence (one batched select).  mode
    "single": all sequences on this GPU; "split": sequence i on rank i % world,
    each rank one batched decode of its own sequences per step; "tp": every
    rank decodes all of them through the tensor-parallel path, selecting by
    the global argmax over the vocab-sharded logits.  A step is the batched
    decode_transition plus the batched select with its tokens copied to the
    host, device-timed per step, max over ranks; the transition alone is
    reported beside it.  The first 3 steps warm up.  The CPU oracle's
    4-sequence subset is checked token for token."""
    lens = [128 + (x % 3969) for x in lcg_ids(args.batch, 1 << 30, SEED + 7)]
    mine = [i for i in range(args.batch) if mode != "split" or i % world == rank]
    if mode == "tp":
        uid = [rdet.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        model.tp_init(rank, world, uid[0])
        model.tp_shard_logits(True)
    nsteps = args.batch_steps
    seqs = [model.new_sequence(lens[i] + nsteps + 8) for i in mine]
    for sq, i in zip(seqs, mine):
        sq.prefill(lcg_ids(lens[i], t["vocab_size"], SEED + 100 + i))
    toks = rdet.select_batch(model, seqs)
    gen = {i: [] for i in mine}
    step_ms, trans_ms = [], []
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    for step in range(nsteps):
        for i, tk in zip(mine, toks):
            gen[i].append(tk)
        b0, bt, b1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        b0.record(stream)
        rdet.decode_batch(model, seqs, toks)
        bt.record(stream)
        toks = rdet.select_batch(model, seqs)  # tokens to the host (synchronizes)
        b1.record(stream)
        b1.synchronize()
        step_ms.append(b0.elapsed_time(b1))
        trans_ms.append(b0.elapsed_time(bt))
    timed = step_ms[3:] if len(step_ms) > 6 else step_ms
    ttimed = trans_ms[3:] if len(trans_ms) > 6 else trans_ms
    bsec = sum(timed) / 1000
    tsec = sum(ttimed) / 1000
    # fixture check: mismatching and checked sequences, summed over the ranks
    bad = checked = 0
    fx = load_fixtures()
    if fx and "config5" in fx and nsteps >= fx["config5"]["tokens_per_sequence"] and args.batch == fx["config5"]["batch"]:
        n5 = fx["config5"]["tokens_per_sequence"]
        for k, r in fx["config5"]["sequences"].items():
            if int(k) in gen:
                checked += 1
                bad += gen[int(k)][:n5] != r["tokens"]
    if dist:
        tt = torch.tensor([bsec, tsec], dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        bsec, tsec = float(tt[0]), float(tt[1])
        cc = torch.tensor([bad, checked], dtype=torch.int64, device=f"cuda:{local_rank}")
        dist.all_reduce(cc, op=dist.ReduceOp.SUM)
        bad, checked = int(cc[0]), int(cc[1])
        if mode == "tp":  # every rank checked the same sequences
            bad, checked = bad // world, checked // world
    for sq in seqs:
        sq.free()
    par = {"single": "single", "split": f"sequences split over {world} ranks", "tp": f"tp{world}"}[mode]
    return {"sequences": args.batch, "context": f"128 + draw mod 3969 (seeded), mean {sum(lens) // len(lens)}",
            "parallelism": par, "scaling": None if mode == "single" else "strong",
            "steps": nsteps, "timed_steps": len(timed), "tok_s": args.batch * len(timed) / bsec,
            "ms_per_step": 1000 * bsec / len(timed), "transition_ms_per_step": 1000 * tsec / len(ttimed),
            "bit_exact_vs_cpu": (bad == 0) if checked else None, "checked_sequences": checked,
            "note": "greedy: a step is one batched decode_transition plus one batched select_output_token "
                    "with the tokens read back to the host, device-timed (max over ranks); tensor-parallel "
                    "ranks select by the global argmax over vocab-sharded logits ((value, index) pairs); "
                    "the first 3 steps are warm-up; bit_exact_vs_cpu checks the CPU oracle's 4-sequence subset "
                    "(tests/golden/e4b_fixtures.json)"}


def run_ours(args, rank, world, local_rank):
    import torch
    rdet = importlib.import_module("raster-inference_b200")
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device(f"cuda:{local_rank}"))
    cfg = load_config()
    t = cfg["text_config"]
    ctx = args.ctx
    model = rdet.Model.synthetic(cfg, SEED, width=16, device=local_rank, max_prefill=ctx)
    stream = torch.cuda.ExternalStream(model.stream, device=f"cuda:{local_rank}")
    seq = model.new_sequence(ctx + args.warmup + args.steps + 64)
    ids = lcg_ids(ctx, t["vocab_size"], SEED + rank)
    # clocks: sampled from the prefills below through the timed decode region
    # (the decode region alone is shorter than the sampler's 200 ms period)
    clk = ClockSampler(local_rank)
    clk.__enter__()
    # prefill of the 4096-token prompt (the prefill field: median of three
    # prefills on fresh sequences after one untimed prefill)
    prefill_runs = []
    for rep in range(4):
        ps = model.new_sequence(ctx + 8)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        ps.prefill(ids)
        e1.record(stream)
        torch.cuda.synchronize()
        if rep:
            prefill_runs.append(e0.elapsed_time(e1) / 1000)
        ps.free()
    prefill_s = statistics.median(prefill_runs)
    seq.prefill(ids)
    # warm-up (captures the decode graph)
    warm_toks = seq.generate(args.warmup)
    kernels_per_step = seq.kernels_per_step() + 2  # + the two argmax kernels of select
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    toks = seq.generate(args.steps)
    b.record(stream)
    torch.cuda.synchronize()
    clk.__exit__(None, None, None)
    if dist:
        dist.barrier()
    sec = a.elapsed_time(b) / 1000
    if dist:
        tt = torch.tensor([sec, prefill_s], dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        sec, prefill_s = float(tt[0]), float(tt[1])
    value = world * args.steps / sec
    # end to end through the C ABI with host buffers: decode_transition(token
    # from host) + select_output_token (token back to host), every step
    n_e2e = min(args.steps, 32)
    tok = toks[-1]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        seq.decode(tok)
        tok = seq.select()
    e2e_sec = time.perf_counter() - t0
    if dist:
        tt = torch.tensor([e2e_sec], dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_sec = float(tt[0])
    e2e = {"value": world * n_e2e / e2e_sec, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
           "steps": n_e2e}
    # BASELINE config 4 as stated: the 4096-token prompt, then 256 greedy
    # tokens (device-timed generation) checked against the CPU oracle's tokens
    config4 = None
    if args.config4_tokens > 0:
        c4 = model.new_sequence(ctx + args.config4_tokens + 8)
        c4.prefill(lcg_ids(ctx, t["vocab_size"], SEED))
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        c4_toks = c4.generate(args.config4_tokens)
        g1.record(stream)
        torch.cuda.synchronize()
        c4_sec = g0.elapsed_time(g1) / 1000
        fx = load_fixtures()
        exact = None
        if fx and "config4" in fx and ctx == fx["config4"]["prompt_tokens"]:
            ref = fx["config4"]["tokens"]
            n4 = min(len(ref), len(c4_toks))
            exact = c4_toks[:n4] == ref[:n4] and (warm_toks + toks == ref[:args.warmup + len(toks)]
                                                  if rank == 0 else True)
        config4 = {"prompt_tokens": ctx, "tokens": args.config4_tokens, "tok_s": args.config4_tokens / c4_sec,
                   "ms_per_token": 1000 * c4_sec / args.config4_tokens, "bit_exact_vs_cpu": exact,
                   "note": "one rdet_generate of all tokens after a fresh prefill; tokens compared with the CPU "
                           "oracle's (tests/golden/e4b_fixtures.json), as are the timed steps' tokens"}
        c4.free()
    # prefill of one seeded uniform prompt of 512 and of
    # 2048 tokens through all layers (device-timed, kernels already warm)
    # (median of three prefills of the same prompt, each on a fresh sequence)
    prefill_lengths = {}
    for plen in (512, 2048):
        pids = lcg_ids(plen, t["vocab_size"], SEED + 11 + plen)
        runs = []
        for _ in range(3):
            ps = model.new_sequence(plen + 8)
            p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            p0.record(stream)
            ps.prefill(pids)
            p1.record(stream)
            torch.cuda.synchronize()
            runs.append(p0.elapsed_time(p1) / 1000)
            ps.free()
        psec = statistics.median(runs)
        ops = prefill_int8_ops(cfg, plen)
        prefill_lengths[str(plen)] = {"tok_s": plen / psec, "seconds": psec, "runs": 3,
                                      "int8_util": ops / psec / INT8_PEAK_OPS,
                                      "int8_util_note": "whole prefill: the tensor-core GEMMs' and attention's int8 "
                                                        "ops / prefill time / 4.5 POPS nominal dense int8"}
    # batched ragged decode: 64 sequences, prompt lengths
    # 128 + draw % 3969 (seeded), greedy: one batched decode_transition per
    # step, then select_output_token for every sequence
    batched = batched_tp = None
    if args.batch > 0:
        # N > 1: "split" gives each rank its share of the 64 sequences (no
        # collective: sequences are independent), then "tp" decodes all 64 on
        # every rank with the tensor-parallel path (rdet_tp_init); both are
        # strong scaling of the same batch.  N = 1: one unsharded run.
        batched = batched_run(args, torch, rdet, dist, model, stream, t, rank, world, local_rank,
                              "split" if world > 1 else "single")
        if world > 1:
            batched_tp = batched_run(args, torch, rdet, dist, model, stream, t, rank, world, local_rank, "tp")
    # roofline of the dominant kernel (det GEMV)
    per, gbs, bytes_per_launch, sec_per_launch, gemv_exact = gemv_roofline(torch, rdet, cfg, local_rank,
                                                                            check=(rank == 0))
    peak, peak_kind = peaks()
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "gemv_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            ratio = json.load(f).get("dram_to_algorithmic_bytes")
        if ratio:
            traffic = ratio * bytes_per_launch
    weight_bytes = model.weight_bytes
    step_bytes = decode_step_bytes(cfg, ctx)
    step_frac = {"bytes_per_step": step_bytes, "achieved_gbs": step_bytes / (sec / args.steps) / 1e9,
                 "frac": step_bytes / (sec / args.steps) / 1e9 / peaks()[0]}
    if dist:
        dist.barrier()
    if rank != 0:
        seq.free()
        model.close()
        if dist:
            dist.destroy_process_group()
        return
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * sec / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int64",
        "data": "synthetic (seeded random-init i16 weights of the E4B stand-in shape; seeded uniform prompt ids)",
        "config": {"workload": "det greedy decode, batch 1, context 4096, E4B stand-in (config 4)",
                   "model": "gemma-4-e4b-text-standin", "context": ctx, "global_batch": world,
                   "parallelism": f"replicas{world}", "l2": "inputs larger than L2 (all weights streamed every step)",
                   "weight_bytes_hbm": weight_bytes},
        "prefill": {"tokens": ctx, "tok_s": ctx / prefill_s, "seconds": prefill_s,
                    "int8_util": prefill_int8_ops(cfg, ctx) / prefill_s / INT8_PEAK_OPS},
        "prefill_config3": prefill_lengths,
        "config4": config4,
        "e2e": e2e,
        "batched_decode": batched,
        "batched_decode_tp": batched_tp,
        "gpu_launches": kernels_per_step * args.steps,
        "roofline": {"bound": "hbm", "kernel": "rdet::gemv3_kernel", "achieved": gbs, "peak": peak,
                     "unit": "GB/s", "frac": gbs / peak, "peak_kind": peak_kind,
                     "traffic": traffic, "algorithmic_bytes_per_launch": bytes_per_launch,
                     "us_per_launch": sec_per_launch * 1e6,
                     "per_shape_gbs": {k: round(v["gbs"], 1) for k, v in per.items()},
                     "per_shape_frac": {k: round(v["gbs"] / peak, 3) for k, v in per.items()},
                     "step_frac": step_frac,
                     "activations": "N(0,1) quantized with f32_to_act (config 2)",
                     "bit_exact_vs_cpu": gemv_exact},
        "clocks": clk.summary(),
    }
    if world == 1:
        line["config1"] = config1_routines(rdet)
    if world == 1 and not args.no_cpu_baseline:
        cores = host_cores()
        times, single, _ = cpu_decode_rate(cfg, ctx, 4, cores, single_thread_steps=3)
        line["cpu_baseline"] = {"value": 3 / sum(times[1:]), "unit": "tok/s", "cores": cores, "kind": "port",
                                "sample": f"3 greedy decode steps (after 1 warm-up) at context {ctx}, seeded synthetic "
                                          f"KV cache, E4B stand-in, {cores} threads, {cpu_model()}",
                                "single_thread": {"value": len(single) / sum(single), "unit": "tok/s", "cores": 1,
                                                  "sample": f"{len(single)} greedy decode steps on one thread, same "
                                                            f"model and cache"}}
    print(json.dumps(line), flush=True)
    seq.free()
    model.close()
    if dist:
        dist.destroy_process_group()


def run_trace_case(args):
    """Cost of a checkpoint-traced run at E4B shape: the det trace of a
    --ctx-token prompt and 2 greedy tokens (every committed checkpoint from
    input.embedding to decode.transition_finalize, per-layer prefill
    commitments and the KV-prefix commitments included), wall-clock through
    the C ABI, beside the same prefill and decode without commitments."""
    import torch
    rdet = importlib.import_module("raster-inference_b200")
    trace = importlib.import_module("raster-inference_b200.trace")
    cfg = load_config()
    t = cfg["text_config"]
    ctx = args.ctx
    ids = lcg_ids(ctx, t["vocab_size"], SEED)
    out = {"case": "checkpoint trace", "prompt_tokens": ctx, "new_tokens": 2}
    for flag in (False, True):
        model = rdet.Model.synthetic(cfg, SEED, width=16, device=0, max_prefill=ctx, layer_commitments=flag)
        for rep in range(2):  # the first pass warms kernels, staging and workers
            seq = model.new_sequence(ctx + 8)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            if flag:
                spent = {}
                backend = trace.SeqBackend(seq)

                def timed(name, fn):
                    def call(*a):
                        c0 = time.perf_counter()
                        r = fn(*a)
                        spent[name] = spent.get(name, 0.0) + time.perf_counter() - c0
                        return r
                    return call

                for name in ("prefill", "select", "decode", "embedding_commitment", "hidden_commitment",
                             "logits_commitment", "layer_output_commitment", "kv_commitment",
                             "kv_prefix_commitments"):
                    setattr(backend, name, timed(name, getattr(backend, name)))
                tr, gen = trace.run(backend, ids, num_layers=model.L, max_new_tokens=2)
            else:
                seq.prefill(ids)
                gen = seq.generate(2)
            torch.cuda.synchronize()
            sec = time.perf_counter() - t0
            seq.free()
        key = "traced" if flag else "plain"
        out[key] = {"seconds": sec, "generated": gen}
        if flag:
            out[key]["entries"] = len(tr.entries)
            out[key]["entries_sha256"] = hashlib.sha256(json.dumps(tr.entries).encode()).hexdigest()
            out[key]["seconds_by_call"] = {k: round(v, 4) for k, v in spent.items()}
        model.close()
    out["overhead_seconds"] = out["traced"]["seconds"] - out["plain"]["seconds"]
    try:
        with open("/proc/cpuinfo") as f:
            sha_ext = " sha_ni" in f.read()
    except OSError:
        sha_ext = False
    out["sha256_impl"] = "x86 SHA extensions" if sha_ext else "scalar"
    out["host"] = cpu_model()
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config4-tokens", type=int, default=256, help="greedy tokens of the config-4 line (0: skip)")
    ap.add_argument("--batch", type=int, default=64, help="sequences of the batched ragged decode line (0: skip)")
    ap.add_argument("--batch-steps", type=int, default=128, help="greedy steps of the batched line (config 5: 128)")
    ap.add_argument("--kernel-case", choices=["gemv", "attn", "tc", "tcattn", "prefill", "convert", "batch", "batchattn"],
                    help="run a few launches of one kernel at E4B shapes for an ncu capture, then exit")
    ap.add_argument("--time-calls", type=int, default=0,
                    help="with --kernel-case attn: time this many back-to-back calls of each decode-attention entry "
                         "point")
    ap.add_argument("--trace-case", action="store_true",
                    help="time a checkpoint-traced run (commitments on) against a plain one at --ctx, then exit")
    args = ap.parse_args()
    if args.trace_case:
        run_trace_case(args)
        return
    if args.kernel_case:
        run_kernel_case(args)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args, rank)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
