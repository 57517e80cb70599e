"""GPU: the allocation-free decode entry point, gqa_decode_launch_noalloc.

Callers such as an engine that reserves all of HBM for its own KV-cache pool,
or a bare C / cgo / JNI binding without a device allocator, cannot hand the
library a workspace; this entry point keeps its scratch in a fixed 16 MiB
device array instead.  The test calls it through the C ABI twice in a row
(the second call reuses the array the first one left behind) and compares
each output with the workspace-based gqa_decode_launch at the suite's
tolerance, and bit for bit (both run the same kernel, grid and schedule).
The file name sorts last so a stop-at-first-failure run has already run
every other test.
"""

import ctypes
import math

import pytest
import torch

import capi
import cases

pytestmark = pytest.mark.gpu

ATOL = 1e-2
RTOL = 1e-2
SCALE = 1.0 / math.sqrt(128)

_P = ctypes.c_void_p
_I = ctypes.c_int
capi.lib.gqa_decode_launch_noalloc.argtypes = [_P] * 6 + [_I] * 6 + [ctypes.c_float, _P]
capi.lib.gqa_decode_launch_noalloc.restype = _I


def noalloc(q, k, v, bt, sl, scale):
    out = torch.full_like(q, float("nan"))
    rc = capi.lib.gqa_decode_launch_noalloc(
        _P(q.data_ptr()), _P(k.data_ptr()), _P(v.data_ptr()), _P(bt.data_ptr()),
        _P(sl.data_ptr()), _P(out.data_ptr()), q.shape[0], q.shape[1], k.shape[2], k.shape[1],
        bt.shape[1], k.shape[0], scale, capi.stream())
    return rc, out


@pytest.mark.parametrize("which", ["a_base", "config1", "ragged"])
def test_noalloc_matches_workspace_entry_point_twice(which):
    if which == "a_base":
        case = cases.ref_case("a_base", seed=31)
    elif which == "config1":
        case = cases.config1()
    else:
        case = cases.make_case(cases.config4_seq_lens(seed=1, B=24), 32, 8, 16, seed=32,
                               pool_factor=1.0 / 0.9)
    gpu = tuple(t.cuda() for t in case)
    expect = capi.auto(*gpu, SCALE)
    for call in range(2):
        rc, out = noalloc(*gpu, SCALE)
        assert rc == 0, f"call {call}: gqa_decode_launch_noalloc returned {rc}"
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all(), f"call {call}: unwritten or non-finite output"
        assert torch.allclose(out.float(), expect.float(), atol=ATOL, rtol=RTOL), \
            f"call {call}: max-abs {(out.float() - expect.float()).abs().max().item():.3e}"
        # same kernel, grid and schedule as the workspace entry point: same bits
        assert torch.equal(out, expect), f"call {call}: not bit-identical to gqa_decode_launch"
    assert capi.status() == 0


def test_noalloc_rejects_shapes_beyond_the_scratch():
    # 4096 requests x 32 heads need ~70 MB of split state: refused up front.
    q = torch.zeros(4096, 32, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(4, 16, 8, 128, dtype=torch.bfloat16, device="cuda")
    bt = torch.zeros(4096, 1, dtype=torch.int32, device="cuda")
    sl = torch.ones(4096, dtype=torch.int32, device="cuda")
    rc, out = noalloc(q, k, k, bt, sl, SCALE)
    torch.cuda.synchronize()
    assert rc == 1  # cudaErrorInvalidValue, nothing launched
    assert torch.isnan(out.float()).all()
