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
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU: the oracle (C++ restatement of the reference det path) on host cores
# ---------------------------------------------------------------------------
def cpu_decode_rate(cfg, ctx, steps, threads):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O  # CPU baseline only
    O.set_threads(threads)
    t0 = time.perf_counter()
    m = O.Model(None, synthetic=(cfg, SEED, 16))
    s = m.seq()
    s.fill_synthetic(ctx, seed=7)
    setup = time.perf_counter() - t0
    times = []
    tok = 1
    for _ in range(steps):
        t = time.perf_counter()
        _, logits, _ = s.decode(tok, want_layer_hashes=False)
        tok = O.argmax_first(logits)
        times.append(time.perf_counter() - t)
    m.close()
    return times, setup


def run_reference(args, rank):
    if rank != 0:
        return  # the CPU arm runs on rank 0 only
    cfg = load_config()
    cores = host_cores()
    times, _ = cpu_decode_rate(cfg, args.ctx, args.warmup + args.steps, cores)
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


def gemv_roofline(torch, rdet, cfg, device, copies=8, rounds=3):
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
    xs = {k: torch.randint(-(1 << 20), 1 << 20, (s[1],), dtype=torch.int32, device=dev, generator=g)
          for k, s in shapes.items()}
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
    out, tot_b, tot_t = {}, 0.0, 0.0
    for k, (n, kk) in shapes.items():
        ms = statistics.mean(a.elapsed_time(b) / c for a, b, c in per[k])
        b = n * kk * 2 + kk * 4 + n * 4
        out[k] = {"rows": n, "cols": kk, "us": ms * 1000, "gbs": b / (ms * 1e-3) / 1e9}
        tot_b += b
        tot_t += ms * 1e-3
    return out, tot_b / tot_t / 1e9, tot_b / len(shapes), tot_t / len(shapes)


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
    # prefill of the 4096-token prompt (timed for the prefill field)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    seq.prefill(ids)
    e1.record(stream)
    torch.cuda.synchronize()
    prefill_s = e0.elapsed_time(e1) / 1000
    # warm-up (captures the decode graph)
    seq.generate(args.warmup)
    kernels_per_step = seq.kernels_per_step() + 2  # + the two argmax kernels of select
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        toks = seq.generate(args.steps)
        b.record(stream)
        torch.cuda.synchronize()
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
        prefill_lengths[str(plen)] = {"tok_s": plen / psec, "seconds": psec, "runs": 3}
    # batched ragged decode (BASELINE config 5 shape): 64 sequences, prompt
    # lengths 128 + draw % 3969 (seeded), one batched decode_transition per step
    batched = None
    if args.batch > 0:
        bm, bstream = model, stream  # max_prefill (the context) >= the batch rows
        # N > 1: the batch is sharded across the ranks (tensor-parallel, same
        # sequences on every rank): strong scaling of this line
        tp = world > 1
        if tp:
            uid = [rdet.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(uid, src=0)
            bm.tp_init(rank, world, uid[0])
        lens = [128 + (x % 3969) for x in lcg_ids(args.batch, 1 << 30, SEED + 7)]
        seqs = [bm.new_sequence(n + args.batch_steps + 8) for n in lens]
        for i, (sq, n) in enumerate(zip(seqs, lens)):
            sq.prefill(lcg_ids(n, t["vocab_size"], SEED + 100 + i))
        toks = [sq.select() for sq in seqs]
        for _ in range(2):  # warm-up
            rdet.decode_batch(bm, seqs, toks)
            toks = [sq.select() for sq in seqs]
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record(bstream)
        for _ in range(args.batch_steps):
            rdet.decode_batch(bm, seqs, toks)
        b1.record(bstream)
        torch.cuda.synchronize()
        bsec = b0.elapsed_time(b1) / 1000
        if dist:
            tt = torch.tensor([bsec], dtype=torch.float64, device=f"cuda:{local_rank}")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            bsec = float(tt[0])
        batched = {"sequences": args.batch, "context": f"128 + draw mod 3969 (seeded), mean {sum(lens) // len(lens)}",
                   "parallelism": f"tp{world}" if tp else "single", "scaling": "strong" if tp else None,
                   "steps": args.batch_steps, "tok_s": args.batch * args.batch_steps / bsec,
                   "ms_per_step": 1000 * bsec / args.batch_steps,
                   "note": "device-timed batched decode_transition (same token fed back: decode cost does not depend "
                           "on token values)"}
        for sq in seqs:
            sq.free()
    # roofline of the dominant kernel (det GEMV)
    per, gbs, bytes_per_launch, sec_per_launch = gemv_roofline(torch, rdet, cfg, local_rank)
    peak, peak_kind = peaks()
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "gemv_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            ratio = json.load(f).get("dram_to_algorithmic_bytes")
        if ratio:
            traffic = ratio * bytes_per_launch
    weight_bytes = model.weight_bytes
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
        "prefill": {"tokens": ctx, "tok_s": ctx / prefill_s, "seconds": prefill_s},
        "prefill_config3": prefill_lengths,
        "e2e": e2e,
        "batched_decode": batched,
        "gpu_launches": kernels_per_step * args.steps,
        "roofline": {"bound": "hbm", "kernel": "rdet::gemv3_kernel", "achieved": gbs, "peak": peak,
                     "unit": "GB/s", "frac": gbs / peak, "peak_kind": peak_kind,
                     "traffic": traffic, "algorithmic_bytes_per_launch": bytes_per_launch,
                     "us_per_launch": sec_per_launch * 1e6,
                     "per_shape_gbs": {k: round(v["gbs"], 1) for k, v in per.items()}},
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        cores = host_cores()
        times, _ = cpu_decode_rate(cfg, ctx, 2, cores)
        line["cpu_baseline"] = {"value": 1.0 / times[-1], "unit": "tok/s", "cores": cores, "kind": "port",
                                "sample": f"1 greedy decode step (after 1 warm-up) at context {ctx}, seeded synthetic "
                                          f"KV cache, E4B stand-in, {cores} threads, {cpu_model()}"}
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
    ap.add_argument("--batch", type=int, default=64, help="sequences of the batched ragged decode line (0: skip)")
    ap.add_argument("--batch-steps", type=int, default=8)
    ap.add_argument("--kernel-case", choices=["gemv", "attn", "tc", "prefill"],
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
