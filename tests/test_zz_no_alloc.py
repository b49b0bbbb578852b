"""The allocation-free decode attention entry point.

rdet_det_attention_decode_noalloc serves callers that cannot allocate device
memory while they run (HBM fully handed to weights and KV caches, or a fixed
per-step footprint); its scratch is a fixed array inside the library.  This
checks, through the C ABI, that calls in a row give exactly the output of the
CPU oracle's attention_output_into and of the allocating entry point
rdet_det_attention_decode on the same inputs (bit-exact: the tolerance of
every parity test here), that a call leaves the free device memory unchanged,
that a call filling the fixed array to all of its limits at once (16 heads,
head_dim 512, 4096 attended rows) is exact, and that oversized requests are
rejected.  Collected last so that a stop-at-first-failure run has already run
the rest.
"""
import numpy as np
import pytest

import oracle as O  # checker only
from helpers import rdet

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _case(seed, heads, kv_heads, d, cap, position, window):
    rng = np.random.default_rng(seed)
    q = rng.integers(-(1 << 17), 1 << 17, (heads, d), dtype=np.int64).astype(np.int32)
    k = rng.integers(-(1 << 17), 1 << 17, (kv_heads, cap, d), dtype=np.int64).astype(np.int32)
    v = rng.integers(-(1 << 20), 1 << 20, (kv_heads, cap, d), dtype=np.int64).astype(np.int32)
    start = max(0, position + 1 - window) if window else 0
    g = heads // kv_heads
    ref = np.stack([O.attention_one(q[h], k[h // g, start:position + 1], v[h // g, start:position + 1])
                    for h in range(heads)])
    return torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), ref


@pytest.mark.parametrize("calls", [[
    (8, 2, 512, 4400, 4095, 0),
    (4, 2, 256, 800, 700, 512),
    # every limit of the fixed array at once: 16 heads, head_dim 512, 4096 rows
    (16, 4, 512, 4096, 4095, 0),
    # a smaller call after the largest: stale contents of the array must not leak in
    (2, 1, 64, 300, 130, 0),
]])
def test_noalloc_matches_oracle_and_allocating_entry_point(calls):
    for n, (heads, kv_heads, d, cap, position, window) in enumerate(calls):
        q, k, v, oracle_out = _case(100 + n, heads, kv_heads, d, cap, position, window)
        ref = torch.full((heads, d), -1, dtype=torch.int32, device="cuda")
        out = torch.full((heads, d), -2, dtype=torch.int32, device="cuda")
        rdet.det_attention_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), cap, heads, kv_heads, d, position,
                                  window, ref.data_ptr())
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rdet.det_attention_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), cap, heads, kv_heads, d,
                                          position, window, out.data_ptr())
        torch.cuda.synchronize()
        if n > 0:  # the first call may load the library's device module (and its fixed array)
            assert torch.cuda.mem_get_info()[0] == free_before
        got = out.cpu().numpy()
        assert np.array_equal(got, oracle_out), f"call {n}: differs from the oracle"
        assert np.array_equal(got, ref.cpu().numpy()), f"call {n}: differs from rdet_det_attention_decode"


def test_noalloc_rejects_sizes_beyond_its_limits():
    q, k, v, _ = _case(7, 8, 2, 64, 5000, 4999, 512)
    out = torch.zeros((8, 64), dtype=torch.int32, device="cuda")
    with pytest.raises(rdet.RdetError) as e:
        rdet.det_attention_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), 5000, 8, 2, 64, 4999, 0,
                                          out.data_ptr())
    assert e.value.code == -6 and "4096" in e.value.msg
    # a window keeps the attended rows within the limit
    rdet.det_attention_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), 5000, 8, 2, 64, 4999, 512,
                                      out.data_ptr())
    torch.cuda.synchronize()
