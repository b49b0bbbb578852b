"""Tensor-parallel batched decode (rdet_tp_init): sharded results equal the
unsharded batched decode bit for bit.  World size 1 runs on one GPU (every
slice is the whole matrix, exercising the sharded code path); world size 2
runs as two child processes on two GPUs and is skipped on a one-GPU box."""
import os
import subprocess
import sys

import numpy as np
import pytest

from helpers import lcg_ids, mini_config, rdet, write_model

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def tp_config():
    # E4B head geometry on a narrow model; dims divide by 2 for the 2-rank test
    return mini_config(hidden_size=256, intermediate_size=512, num_attention_heads=8, num_key_value_heads=2,
                       head_dim=256, global_head_dim=512, sliding_window=512, hidden_size_per_layer_input=32,
                       num_hidden_layers=4, num_kv_shared_layers=1, vocab_size=300,
                       layer_types=["sliding_attention", "full_attention", "sliding_attention", "sliding_attention"])


def run_pair(d, lens, steps, rank, world, uid, device=0, exchange=None, shard_logits=False):
    """Decodes the same ragged batch on a sharded and an unsharded context of
    one device and compares them step by step.  exchange: a function that
    takes this rank's NVLink-reduction blob and returns all ranks' blobs in
    rank order (the sharded context then reduces over NVLink, not NCCL).
    shard_logits: the sharded context selects by the global argmax over the
    ranks' (value, index) pairs and never assembles the logit rows."""
    sharded = rdet.Model.open(d, device=device, max_prefill=max(max(lens), len(lens)))
    plain = rdet.Model.open(d, device=device, max_prefill=max(max(lens), len(lens)))
    sharded.tp_init(rank, world, uid)
    if exchange is not None:
        sharded.tp_ipc_connect(exchange(sharded.tp_ipc_export(len(lens)), "blob"))
    if shard_logits:
        sharded.tp_shard_logits(True)
    assert sharded.tp_world == world and plain.tp_world == 1
    a = [sharded.new_sequence(n + steps + 4) for n in lens]
    b = [plain.new_sequence(n + steps + 4) for n in lens]
    for i, n in enumerate(lens):
        ids = lcg_ids(n, 300, 200 + i)
        a[i].prefill(ids)
        b[i].prefill(ids)
    for step in range(steps):
        toks = [s.select() for s in b]
        assert toks == rdet.select_batch(sharded, a), step
        rdet.decode_batch(sharded, a, toks)
        rdet.decode_batch(plain, b, toks)
        for i, (x, y) in enumerate(zip(a, b)):
            if shard_logits:
                with pytest.raises(rdet.RdetError, match="vocab-sharded"):
                    x.read(rdet.BUF_LOGITS)
            else:
                assert np.array_equal(x.read(rdet.BUF_LOGITS), y.read(rdet.BUF_LOGITS)), (step, i)
            assert x.commitment(rdet.BUF_HIDDEN) == y.commitment(rdet.BUF_HIDDEN), (step, i)
            assert x.commitment(rdet.BUF_KV) == y.commitment(rdet.BUF_KV), (step, i)
    assert rdet.select_batch(sharded, a) == [s.select() for s in b]
    if exchange is not None:
        # no rank frees its reduction buffers while another may still read them
        torch.cuda.synchronize(device)
        exchange(b"done", "done")


LENS = [5 + (97 * i) % 640 for i in range(34)]


def test_tp_world1_matches_unsharded():
    d = write_model(tp_config(), seed=61)
    run_pair(d, LENS, 3, 0, 1, rdet.nccl_unique_id())


def test_tp_world1_nvlink_reduction_matches_unsharded():
    # one rank: the reduction buffers, flags and fused row kernels without peers
    d = write_model(tp_config(), seed=63)
    run_pair(d, LENS, 3, 0, 1, rdet.nccl_unique_id(), exchange=lambda blob, tag: [blob])


def test_tp_world1_sharded_logits_select_matches_unsharded():
    # the global argmax over (value, index) pairs of the vocab rows
    d = write_model(tp_config(), seed=65)
    run_pair(d, LENS, 3, 0, 1, rdet.nccl_unique_id(), shard_logits=True)


def test_tp_ipc_export_needs_tp_init():
    d = write_model(tp_config(), seed=64)
    m = rdet.Model.open(d, max_prefill=8)
    with pytest.raises(rdet.RdetError, match="rdet_tp_init"):
        m.tp_ipc_export(8)
    m.close()


CHILD = r"""
import os, sys
root = sys.argv[1]
sys.path[:0] = [os.path.join(root, "tests"), os.path.join(root, "tests", "golden"), os.path.join(root, "oracle"), root]
import test_gpu_tp as T
rank, world, uid, d = int(sys.argv[2]), int(sys.argv[3]), bytes.fromhex(sys.argv[4]), sys.argv[5]
xdir = sys.argv[6] if len(sys.argv) > 6 and sys.argv[6] != "-" else None
shard = len(sys.argv) > 7 and sys.argv[7] == "shard"

def exchange(blob, tag):
    # blobs through files in a shared folder; bounded wait for the other ranks
    import time
    path = lambda r: os.path.join(xdir, f"{tag}{r}")
    open(path(rank) + ".tmp", "wb").write(blob)
    os.replace(path(rank) + ".tmp", path(rank))
    for _ in range(1200):
        if all(os.path.exists(path(r)) for r in range(world)):
            return [open(path(r), "rb").read() for r in range(world)]
        time.sleep(0.05)
    raise RuntimeError("the other ranks' " + tag + " files did not arrive")

T.run_pair(d, T.LENS, 3, rank, world, uid, device=rank, exchange=exchange if xdir else None, shard_logits=shard)
print("TP-OK", rank)
"""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("nvlink,shard", [(False, False), (True, False), (True, True)])
def test_tp_two_gpus_match_unsharded(nvlink, shard, tmp_path):
    d = write_model(tp_config(), seed=62)
    uid = rdet.nccl_unique_id().hex()
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    extra = [str(tmp_path) if nvlink else "-", "shard" if shard else "plain"]
    procs = [subprocess.Popen(["timeout", "-k", "10", "300", sys.executable, "-c", CHILD, root, str(r), "2", uid, d]
                              + extra, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, env=env)
             for r in range(2)]
    outs = [p.communicate(timeout=360)[0] for p in procs]
    for r, (p, out) in enumerate(zip(procs, outs)):
        assert p.returncode == 0 and f"TP-OK {r}" in out, out[-3000:]
