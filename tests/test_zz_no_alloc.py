"""The allocation-free decode attention entry point.

rdet_det_attention_decode_noalloc serves callers that cannot allocate device
memory while they run (HBM fully handed to weights and KV caches, or a fixed
per-step footprint); its scratch is a fixed array inside the library.  This
checks, through the C ABI, that two calls in a row give exactly the output of
the allocating entry point rdet_det_attention_decode on the same inputs
(bit-exact: the tolerance of every parity test here), that a call leaves the
free device memory unchanged, and that oversized requests are rejected.
Collected last so that a stop-at-first-failure run has already run the rest.
"""
import numpy as np
import pytest

from helpers import rdet

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _case(seed, heads, kv_heads, d, cap):
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-(1 << 17), 1 << 17, (heads, d), dtype=torch.int32, generator=g).cuda()
    k = torch.randint(-(1 << 17), 1 << 17, (kv_heads, cap, d), dtype=torch.int32, generator=g).cuda()
    v = torch.randint(-(1 << 20), 1 << 20, (kv_heads, cap, d), dtype=torch.int32, generator=g).cuda()
    return q, k, v


@pytest.mark.parametrize("calls", [[(8, 2, 512, 4400, 4095, 0), (4, 2, 256, 800, 700, 512)]])
def test_noalloc_matches_allocating_entry_point_twice(calls):
    for n, (heads, kv_heads, d, cap, position, window) in enumerate(calls):
        q, k, v = _case(100 + n, heads, kv_heads, d, cap)
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
        assert torch.equal(out, ref), f"call {n}"


def test_noalloc_rejects_sizes_beyond_its_limits():
    q, k, v = _case(7, 8, 2, 64, 5000)
    out = torch.zeros((8, 64), dtype=torch.int32, device="cuda")
    with pytest.raises(rdet.RdetError) as e:
        rdet.det_attention_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), 5000, 8, 2, 64, 4999, 0,
                                          out.data_ptr())
    assert e.value.code == -6 and "4096" in e.value.msg
    # a window keeps the attended rows within the limit
    rdet.det_attention_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), 5000, 8, 2, 64, 4999, 512,
                                      out.data_ptr())
    torch.cuda.synchronize()
