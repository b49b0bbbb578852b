"""The tensor-parallel decomposition on the CPU with two gloo ranks.

The batched decode's tensor-parallel step (rdet_tp_init, csrc/runtime.cu
tp_init / tp_linear_reduce) gives rank r query heads [r Hq/N, (r+1) Hq/N), MLP
gate/up rows F/N and vocab rows V/N, with the matching column slices of o and
down.  A column slice yields the exact pre-requantize i64 partial sum over its
K range; one all-reduce (int64 sum) completes it and requantize gives the
replicated row; vocab rows are all-gathered before argmax_first.  This test
replays that plan for one attention-output projection, one GELU MLP and the
logits, each rank in its own process over gloo, and checks every result bit
for bit against the unsharded computation of the oracle.  It also replays the
vocab-sharded selection (rdet_tp_shard_logits): each rank's first max per row
as a (value, global index) pair, the pairs all-gathered and reduced, equal to
argmax_first over the whole row, ties across the shards included, and the
max-over-ranks step time that bench.py reports for N > 1."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, HQ, D, F, V, S = 64, 4, 16, 96, 200, 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights():
    rng = np.random.default_rng(2024)
    wo = rng.integers(-32768, 32768, (H, HQ * D), dtype=np.int64).astype(np.int16)
    wg = rng.integers(-32768, 32768, (F, H), dtype=np.int64).astype(np.int16)
    wu = rng.integers(-32768, 32768, (F, H), dtype=np.int64).astype(np.int16)
    wd = rng.integers(-32768, 32768, (H, F), dtype=np.int64).astype(np.int16)
    wl = rng.integers(-32768, 32768, (V, H), dtype=np.int64).astype(np.int16)
    attn = rng.integers(-(1 << 22), 1 << 22, (S, HQ * D), dtype=np.int64).astype(np.int32)
    x = rng.integers(-(1 << 20), 1 << 20, (S, H), dtype=np.int64).astype(np.int32)
    return wo, wg, wu, wd, wl, attn, x


def _linear(O, x, w):
    """The oracle's det linear: requantize(sum_k x[s, k] w[n, k])."""
    L = O.lib()
    x = np.ascontiguousarray(x, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.int16)
    y = np.empty((x.shape[0], w.shape[0]), dtype=np.int32)
    L.dor_linear(x.ctypes.data, x.shape[0], w.ctypes.data, 16, w.shape[0], w.shape[1], y.ctypes.data)
    return y


def _partial(x, w):
    """Exact i64 partial sums of a column slice (wrapping, like the kernels)."""
    return x.astype(np.int64) @ w.astype(np.int64).T


def _requantize(O, a):
    L = O.lib()
    return np.array([L.dor_requantize(int(v)) for v in a.ravel()], dtype=np.int32).reshape(a.shape)


def _gelu_mul(O, g, u):
    L = O.lib()
    return np.array([L.dor_mul_sat(L.dor_gelu(int(a)), int(b)) for a, b in zip(g.ravel(), u.ravel())],
                    dtype=np.int32).reshape(g.shape)


def _rank(rank, world, port):
    import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        wo, wg, wu, wd, wl, attn, x = _weights()
        hql, fl, vl = HQ // world, F // world, V // world
        # o projection: this rank's query heads are a column slice of o
        c0, c1 = rank * hql * D, (rank + 1) * hql * D
        part = torch.from_numpy(_partial(attn[:, c0:c1], wo[:, c0:c1]))
        dist.all_reduce(part, op=dist.ReduceOp.SUM)
        o = _requantize(O, part.numpy())
        assert np.array_equal(o, _linear(O, attn, wo))
        # MLP: gate/up rows F/N, GELU(gate)*up on the slice, down column slice
        r0, r1 = rank * fl, (rank + 1) * fl
        act = _gelu_mul(O, _linear(O, x, wg[r0:r1]), _linear(O, x, wu[r0:r1]))
        part = torch.from_numpy(_partial(act, wd[:, r0:r1]))
        dist.all_reduce(part, op=dist.ReduceOp.SUM)
        mlp = _requantize(O, part.numpy())
        full_act = _gelu_mul(O, _linear(O, x, wg), _linear(O, x, wu))
        assert np.array_equal(mlp, _linear(O, full_act, wd))
        # logits: vocab rows V/N, all-gathered, then argmax_first per row
        mine = torch.from_numpy(_linear(O, x, wl[rank * vl:(rank + 1) * vl]))
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        logits = torch.cat(parts, dim=1).numpy()
        full = _linear(O, x, wl)
        assert np.array_equal(logits, full)
        for s in range(S):
            assert O.argmax_first(list(logits[s])) == O.argmax_first(list(full[s]))
        # vocab-sharded selection: pairs instead of rows, lowest index on ties
        rows = np.array(full, dtype=np.int64)
        top = int(rows.max()) + 1
        rows[0, [3, vl + 5]] = top            # tie across the shard boundary: rank 0's index wins
        rows[1, [vl + 7, vl + 2]] = top       # tie inside the last shard
        rows[2, :] = -7                       # every value tied: index 0
        rows = rows.astype(np.int32)
        mine = rows[:, rank * vl:(rank + 1) * vl]
        pairs = torch.tensor([[int(r.max()), rank * vl + int(np.argmax(r))] for r in mine], dtype=torch.int64)
        got = [torch.empty_like(pairs) for _ in range(world)]
        dist.all_gather(got, pairs)
        for s in range(S):
            cand = sorted((-int(g[s, 0]), int(g[s, 1])) for g in got)
            assert cand[0][1] == O.argmax_first(list(rows[s]))
        assert O.argmax_first(list(rows[0])) == 3 and O.argmax_first(list(rows[2])) == 0
        # bench.py's N > 1 timing: every rank takes the maximum of the ranks' times
        t = torch.tensor([1.5 + rank, 0.25 * (world - rank)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        assert t.tolist() == [1.5 + world - 1, 0.25 * world]
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_plan_is_bit_exact_on_two_gloo_ranks():
    mp.start_processes(_rank, args=(2, _free_port()), nprocs=2, join=True, start_method="spawn")


def test_unsharded_reference_is_sane():
    # the single-process check the ranks build on: a column split of the
    # i64 sums recombines exactly
    import oracle as O
    wo, _, _, _, _, attn, _ = _weights()
    halves = _partial(attn[:, :32], wo[:, :32]) + _partial(attn[:, 32:], wo[:, 32:])
    assert np.array_equal(_requantize(O, halves), _linear(O, attn, wo))
