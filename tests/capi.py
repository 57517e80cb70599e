"""Test-side ctypes calls of the C ABI (include/gqa_decode.h).

Every output and split workspace is pre-filled with NaN, so a row the
kernels fail to write can never pass a comparison by inheriting stale
memory.  Launches go on torch's current stream.
"""

import ctypes

import torch

import binding  # loads libgqa_decode_b200.so globally (same device globals)

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_Z = ctypes.c_size_t

lib = ctypes.CDLL(binding.LIB_PATH)
for _name in ("gqa_decode_v0_launch", "gqa_decode_v1_launch"):
    getattr(lib, _name).argtypes = [_P] * 6 + [_I] * 5 + [_F, _P]
    getattr(lib, _name).restype = None
lib.gqa_decode_v2_launch.argtypes = [_P] * 6 + [_I] * 5 + [_F, _I, _P, _P, _P, _P]
lib.gqa_decode_v2_launch.restype = None
lib.gqa_decode_last_error.restype = _I
lib.gqa_decode_launch.argtypes = [_P] * 6 + [_I] * 6 + [_F, _I, _P, _Z, _P]
lib.gqa_decode_launch.restype = _I
lib.gqa_decode_partial_launch.argtypes = [_P] * 8 + [_I] * 6 + [_F, _P, _Z, _P]
lib.gqa_decode_partial_launch.restype = _I
lib.gqa_decode_merge_states.argtypes = [_P, _P, _P, _I, _I, _P, _P]
lib.gqa_decode_merge_states.restype = _I
lib.gqa_decode_workspace_bytes.argtypes = [_I, _I, _I, _I]
lib.gqa_decode_workspace_bytes.restype = _Z
lib.gqa_decode_get_status.argtypes = [ctypes.POINTER(_I), _I]
lib.gqa_decode_get_status.restype = _I
lib.gqa_decode_selftest_wait_timeout.argtypes = [_I, _P]
lib.gqa_decode_selftest_wait_timeout.restype = _I


def stream():
    return _P(torch.cuda.current_stream().cuda_stream)


def _dims(q, k, bt):
    return q.shape[0], q.shape[1], k.shape[2], k.shape[1], bt.shape[1]


def _nan_like(q):
    return torch.full_like(q, float("nan"))


def _ptrs(*ts):
    return [_P(t.data_ptr()) for t in ts]


def v0(q, k, v, bt, sl, scale):
    out = _nan_like(q)
    B, Hq, Hkv, bs, mb = _dims(q, k, bt)
    lib.gqa_decode_v0_launch(*_ptrs(q, k, v, bt, sl, out), B, Hq, Hkv, bs, mb, scale, stream())
    assert lib.gqa_decode_last_error() == 0
    return out


def v1(q, k, v, bt, sl, scale):
    out = _nan_like(q)
    B, Hq, Hkv, bs, mb = _dims(q, k, bt)
    lib.gqa_decode_v1_launch(*_ptrs(q, k, v, bt, sl, out), B, Hq, Hkv, bs, mb, scale, stream())
    assert lib.gqa_decode_last_error() == 0
    return out


def v2(q, k, v, bt, sl, scale, num_splits=8):
    out = _nan_like(q)
    B, Hq, Hkv, bs, mb = _dims(q, k, bt)
    ws_acc = torch.full((B, Hq, num_splits, 128), float("nan"), device=q.device)
    ws_m = torch.full((B, Hq, num_splits), float("nan"), device=q.device)
    ws_l = torch.full((B, Hq, num_splits), float("nan"), device=q.device)
    lib.gqa_decode_v2_launch(*_ptrs(q, k, v, bt, sl, out), B, Hq, Hkv, bs, mb, scale,
                             num_splits, *_ptrs(ws_acc, ws_m, ws_l), stream())
    assert lib.gqa_decode_last_error() == 0
    return out


def workspace(q, k, num_splits):
    nbytes = lib.gqa_decode_workspace_bytes(q.shape[0], q.shape[1], k.shape[2], num_splits)
    return binding.workspace(q.device, nbytes), nbytes


def auto(q, k, v, bt, sl, scale, num_splits=0, check_blocks=True):
    out = _nan_like(q)
    B, Hq, Hkv, bs, mb = _dims(q, k, bt)
    ws, _ = workspace(q, k, num_splits)
    rc = lib.gqa_decode_launch(*_ptrs(q, k, v, bt, sl, out), B, Hq, Hkv, bs, mb,
                               k.shape[0] if check_blocks else 0, scale, num_splits,
                               _P(ws.data_ptr()), ws.numel(), stream())
    assert rc == 0, f"gqa_decode_launch returned {rc}"
    return out


def partial(q, k, v, bt, sl, scale):
    B, Hq, Hkv, bs, mb = _dims(q, k, bt)
    m = torch.full((B, Hq), float("nan"), device=q.device)
    l = torch.full((B, Hq), float("nan"), device=q.device)
    acc = torch.full((B, Hq, 128), float("nan"), device=q.device)
    ws, _ = workspace(q, k, 0)
    rc = lib.gqa_decode_partial_launch(*_ptrs(q, k, v, bt, sl, m, l, acc), B, Hq, Hkv, bs, mb,
                                       k.shape[0], scale, _P(ws.data_ptr()), ws.numel(),
                                       stream())
    assert rc == 0, f"gqa_decode_partial_launch returned {rc}"
    return m, l, acc


def merge(m, l, acc):
    n, rows = m.shape
    out = torch.full((rows, 128), float("nan"), dtype=torch.bfloat16, device=m.device)
    rc = lib.gqa_decode_merge_states(*_ptrs(m, l, acc), n, rows, _P(out.data_ptr()), stream())
    assert rc == 0
    return out


def status(clear=True):
    s = _I(0)
    assert lib.gqa_decode_get_status(ctypes.byref(s), 1 if clear else 0) == 0
    return s.value


KERNELS = {"v0": v0, "v1": v1, "v2": v2, "auto": auto}
