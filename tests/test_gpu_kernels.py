"""det GEMV / linear kernels vs the oracle, bit-exact, through the C ABI on
device buffers (torch is used only to hold device memory)."""
import numpy as np
import pytest

import oracle as O
from helpers import rdet

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

I32_MIN, I32_MAX = -2**31, 2**31 - 1


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rand_w(rng, rows, cols, width, adversarial=False):
    if width == 16:
        w = rng.integers(-32768, 32768, (rows, cols), dtype=np.int64).astype(np.int16)
        if adversarial:
            w.flat[::3] = -32768
            w.flat[1::3] = 32767
        return w
    bound = (2**31 - 1) // cols
    w = rng.integers(-bound, bound + 1, (rows, cols), dtype=np.int64).astype(np.int32)
    if adversarial:
        w.flat[::2] = bound
    return w


def rand_x(rng, n, adversarial=False):
    x = rng.integers(I32_MIN, I32_MAX, n, dtype=np.int64).astype(np.int32) if adversarial else \
        rng.normal(0, 65536 * 4, n).astype(np.int64).clip(I32_MIN, I32_MAX).astype(np.int32)
    if adversarial:
        x[::5] = I32_MIN
        x[1::5] = I32_MAX
    return x


SHAPES = [(1, 8), (7, 4), (33, 24), (300, 12), (129, 1000), (513, 2560), (2048, 2560), (2560, 10240)]


@pytest.mark.parametrize("width", [16, 32])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("adv", [False, True])
def test_gemv_bit_exact(width, shape, adv):
    rng = np.random.default_rng(hash((width, shape, adv)) & 0xFFFF)
    rows, cols = shape
    w = rand_w(rng, rows, cols, width, adv)
    x = rand_x(rng, cols, adv)
    y = torch.zeros(rows, dtype=torch.int32, device="cuda")
    wd, xd = dev(w), dev(x)
    rdet.det_gemv(xd.data_ptr(), wd.data_ptr(), width, rows, cols, y.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy(), O.gemv(x, w))


@pytest.mark.parametrize("width", [16, 32])
@pytest.mark.parametrize("S,rows,cols", [
    (1, 64, 64), (5, 70, 33), (64, 128, 256), (130, 96, 520), (17, 2560, 512),
    # tensor-core path (>= 32 rows, i16, cols % 16 == 0): one partial tile, odd
    # row counts, several M and N tiles, K across many stages and the longest K
    (32, 16, 16), (33, 97, 48), (200, 2560, 512), (257, 300, 2560), (129, 193, 1024), (96, 256, 10240),
    # at most 64 rows: the swapped-operand kernel (weights as the 128-row MMA
    # operand), with K split across SMs and with one K range
    (64, 2560, 2560), (48, 1000, 4096), (64, 4096, 256),
    # more than 128 rows: CTA pairs (256-token tiles, the weight planes split
    # across the pair), a partial second half-tile, both tile orders (more
    # activation than weight bytes, and fewer)
    (1000, 2048, 2560), (777, 96, 4096), (2048, 2560, 10240)])
def test_linear_bit_exact(width, S, rows, cols):
    rng = np.random.default_rng(S * 1000 + rows + width)
    w = rand_w(rng, rows, cols, width, True)
    X = np.stack([rand_x(rng, cols, adversarial=(i % 2 == 0)) for i in range(S)])
    Y = torch.zeros((S, rows), dtype=torch.int32, device="cuda")
    Xd, wd = dev(X), dev(w)  # keep the device buffers alive across the launch
    rdet.det_linear(Xd.data_ptr(), S, wd.data_ptr(), width, rows, cols, Y.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(Y.cpu().numpy(), O.linear(X, w))


def test_gemv_rejects_bad_width():
    with pytest.raises(rdet.RdetError):
        rdet.det_gemv(1, 1, 8, 4, 4, 1)


def attention_case(rng, heads, kv_heads, d, cap, position, window, scale=1 << 17):
    q = rng.integers(-scale, scale, (heads, d), dtype=np.int64).astype(np.int32)
    k = rng.integers(-scale, scale, (kv_heads, cap, d), dtype=np.int64).astype(np.int32)
    v = rng.integers(-scale * 8, scale * 8, (kv_heads, cap, d), dtype=np.int64).astype(np.int32)
    start = max(0, position + 1 - window) if window else 0
    g = heads // kv_heads
    ref = np.stack([O.attention_one(q[h], k[h // g, start:position + 1], v[h // g, start:position + 1])
                    for h in range(heads)])
    return q, k, v, ref


@pytest.mark.parametrize("heads,kv_heads,d,cap,position,window", [
    (2, 1, 2, 16, 0, 0), (4, 2, 16, 100, 57, 8), (8, 2, 256, 600, 599, 512), (8, 2, 512, 4400, 4351, 0),
    (8, 1, 64, 300, 130, 0), (3, 3, 48, 70, 69, 1),
    # fewer window rows than cluster CTAs; a head dim below the 16-byte chunk
    # grid; many query heads (several waves of clusters); the first tiles of a
    # sliding window
    (8, 2, 512, 64, 5, 0), (4, 4, 192, 2000, 1999, 0), (16, 4, 128, 3100, 3099, 0), (8, 2, 256, 40, 20, 512)])
def test_attention_decode_bit_exact(heads, kv_heads, d, cap, position, window):
    rng = np.random.default_rng(position + d)
    q, k, v, ref = attention_case(rng, heads, kv_heads, d, cap, position, window)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = torch.zeros((heads, d), dtype=torch.int32, device="cuda")
    rdet.det_attention_decode(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), cap, heads, kv_heads, d, position, window,
                              out.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), ref)


def test_attention_decode_ties_keep_first_max():
    # equal scores everywhere: softmax residual goes to the first row of the window
    heads, kv_heads, d, cap, position, window = 2, 1, 8, 300, 260, 200
    q = np.zeros((heads, d), dtype=np.int32)
    k = np.ones((kv_heads, cap, d), dtype=np.int32)
    v = np.arange(kv_heads * cap * d, dtype=np.int32).reshape(kv_heads, cap, d)
    start = position + 1 - window
    ref = np.stack([O.attention_one(q[h], k[0, start:position + 1], v[0, start:position + 1]) for h in range(heads)])
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = torch.zeros((heads, d), dtype=torch.int32, device="cuda")
    rdet.det_attention_decode(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), cap, heads, kv_heads, d, position, window,
                              out.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), ref)


FRESH_PROCESS_SCRIPT = r"""
import os, sys, numpy as np, torch
root = sys.argv[2]
sys.path[:0] = [sys.argv[1], os.path.join(root, "tests", "golden"), os.path.join(root, "oracle"), root]
from helpers import rdet
import oracle as O
from test_gpu_kernels import attention_case, dev
rng = np.random.default_rng(5)
for heads, kv, d, cap, pos, win in [(8, 2, 256, 700, 650, 512), (8, 2, 512, 300, 299, 0)]:
    q, k, v, ref = attention_case(rng, heads, kv, d, cap, pos, win)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = torch.zeros((heads, d), dtype=torch.int32, device="cuda")
    rdet.det_attention_decode(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), cap, heads, kv, d, pos, win, out.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), ref), (heads, kv, d, pos, win)
print("FRESH-OK")
"""


def test_kernel_entries_in_a_fresh_process():
    # the kernel-level entry points set up their device on first use: no
    # model needs to have been opened in the process
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    r = subprocess.run([sys.executable, "-c", FRESH_PROCESS_SCRIPT, here, os.path.dirname(here)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "FRESH-OK" in r.stdout, r.stdout + r.stderr


@pytest.mark.parametrize("heads,kv_heads,d,cap,position,window", [(8, 2, 256, 600, 599, 512), (8, 2, 512, 300, 299, 0),
                                                                 (2, 1, 64, 50, 40, 0)])
def test_attention_decode_scores_all_int32_min(heads, kv_heads, d, cap, position, window):
    # every score saturates at INT32_MIN, so every row ties: argmax_first picks
    # the first row of the window (det_num/ops.rs:463-478)
    rng = np.random.default_rng(d + position)
    q = np.full((heads, d), I32_MAX, dtype=np.int32)
    k = np.full((kv_heads, cap, d), I32_MIN, dtype=np.int32)
    v = rng.integers(I32_MIN, I32_MAX, (kv_heads, cap, d), dtype=np.int64).astype(np.int32)
    start = max(0, position + 1 - window) if window else 0
    g = heads // kv_heads
    ref = np.stack([O.attention_one(q[h], k[h // g, start:position + 1], v[h // g, start:position + 1])
                    for h in range(heads)])
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = torch.zeros((heads, d), dtype=torch.int32, device="cuda")
    rdet.det_attention_decode(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), cap, heads, kv_heads, d, position, window,
                              out.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("S,rows,cols,edge_row", [(300, 2560, 2560, None), (1000, 960, 4096, None),
                                                  (600, 2048, 2560, 437), (257, 96, 10240, 256)])
def test_linear_activations_within_24_bits_bit_exact(S, rows, cols, edge_row):
    # rows whose values all lie in [-2^23, 2^23) are offset by 2^23 and the CTA
    # pair skips activation limb 3 on tiles made only of such rows; one row at
    # the boundary (2^23 itself) forces the fourth limb on its 256-row tile
    rng = np.random.default_rng(S + rows + cols)
    w = rand_w(rng, rows, cols, 16, True)
    X = rng.integers(-(1 << 23), 1 << 23, (S, cols), dtype=np.int64).astype(np.int32)
    X[0, :4] = [-(1 << 23), (1 << 23) - 1, 0, -1]
    if edge_row is not None:
        X[edge_row, 5] = 1 << 23
    Y = torch.zeros((S, rows), dtype=torch.int32, device="cuda")
    Xd, wd = dev(X), dev(w)
    rdet.det_linear(Xd.data_ptr(), S, wd.data_ptr(), 16, rows, cols, Y.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(Y.cpu().numpy(), O.linear(X, w))
