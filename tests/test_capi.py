"""CPU: the C-ABI library loads, exports every declared entry point, and its
host-only planning functions behave.  No call here touches a GPU."""

import ctypes
import glob
import os
import re

import pytest

import gqa_build as pkg_build

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "gqa_decode.h")


class Plan(ctypes.Structure):
    _fields_ = [("group", ctypes.c_int), ("heads_per_row", ctypes.c_int),
                ("consumer_warps", ctypes.c_int), ("threads", ctypes.c_int),
                ("stages", ctypes.c_int), ("smem_bytes", ctypes.c_int), ("grid", ctypes.c_int),
                ("workspace_bytes", ctypes.c_size_t)]


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(pkg_build.LIB_PATH):
        pkg_build.build_lib()
    L = ctypes.CDLL(pkg_build.LIB_PATH)
    L.gqa_decode_query_plan.argtypes = [ctypes.c_int] * 6 + [ctypes.POINTER(Plan)]
    L.gqa_decode_query_plan.restype = ctypes.c_int
    L.gqa_decode_pick_splits.argtypes = [ctypes.c_int] * 5
    L.gqa_decode_pick_splits.restype = ctypes.c_int
    L.gqa_decode_version.restype = ctypes.c_char_p
    return L


def declared_functions():
    """Every function declared in include/*.h (gqa_decode_*, mla_decode_*, dsa_*)."""
    names = set()
    for h in sorted(glob.glob(os.path.join(REPO, "include", "*.h"))):
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names.update(re.findall(
            r"^\s*(?:const\s+)?[\w]+\s*\*?\s+((?:gqa_decode|mla_decode|dsa)_\w+)\s*\(", text,
            flags=re.M))
    return sorted(names)


def test_header_declares_reference_launchers():
    names = declared_functions()
    for n in ["gqa_decode_v0_launch", "gqa_decode_v1_launch", "gqa_decode_v2_launch"]:
        assert n in names
    assert len(names) >= 13


@pytest.mark.parametrize("name", declared_functions())
def test_symbol_exported(lib, name):
    assert hasattr(lib, name), f"{name} declared in include/*.h but not exported"


def _dynamic_symbols():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", pkg_build.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


# The C++-mangled names of the reference's three launchers as declared in its
# include/gqa_decode.h:6-23 (C++ linkage): (const __nv_bfloat16*) x3,
# (const int*) x2, __nv_bfloat16*, int x5, float, [int, float* x3,] cudaStream_t.
CXX_LAUNCHERS = [
    "_Z20gqa_decode_v0_launchPK13__nv_bfloat16S1_S1_PKiS3_PS_iiiiifP11CUstream_st",
    "_Z20gqa_decode_v1_launchPK13__nv_bfloat16S1_S1_PKiS3_PS_iiiiifP11CUstream_st",
    "_Z20gqa_decode_v2_launchPK13__nv_bfloat16S1_S1_PKiS3_PS_iiiiifiPfS5_S5_P11CUstream_st",
]


def test_declared_symbols_have_c_linkage():
    # extern "C" in include/*.h: the dynamic symbol table holds the plain names.
    syms = _dynamic_symbols()
    for name in declared_functions():
        assert name in syms


def test_reference_launchers_also_have_cxx_linkage():
    # An object compiled against the reference header references these.
    syms = _dynamic_symbols()
    for name in CXX_LAUNCHERS:
        assert name in syms, f"{name} (C++ linkage) not exported"


def test_version(lib):
    assert b"sm_100a" in lib.gqa_decode_version()


def align256(x):
    return (x + 255) // 256 * 256


def plan_bytes(grid, B):
    # balanced-schedule plan: 8 header words + 4 per CTA, and the [B + 1] prefix
    return align256((8 + 4 * grid) * 8) + align256((B + 1) * 8)


def plan(lib, B, Hq, Hkv, ns=0, sms=148, per_sm=1):
    p = Plan()
    rc = lib.gqa_decode_query_plan(B, Hq, Hkv, ns, sms, per_sm, ctypes.byref(p))
    return rc, p


def test_plan_rep_shape(lib):
    rc, p = plan(lib, 32, 32, 8)
    assert rc == 0
    assert p.group == 4 and p.heads_per_row == 8 and p.consumer_warps == 8
    assert p.threads == 288
    assert p.stages == 3
    assert p.smem_bytes <= 227 * 1024
    assert p.grid == 148
    assert p.workspace_bytes == balanced_bytes(148, 32, rows=32, qhr=32)


def balanced_bytes(grid, B, rows, qhr):
    # plan + prefix, row records {first CTA, parts} per row, CTA records
    # {row, parts} per CTA, then m, l, acc for (grid + rows) slots x qhr heads
    slots = grid + rows
    return (plan_bytes(grid, B) + align256(rows * 8) + align256(grid * 8) +
            2 * align256(slots * qhr * 4) + slots * qhr * 128 * 4)


@pytest.mark.parametrize("Hq,Hkv,hg,ncw", [(64, 8, 8, 8), (32, 8, 8, 8), (64, 4, 4, 8),
                                           (128, 8, 4, 8), (32, 1, 1, 4), (8, 8, 8, 8),
                                           (24, 8, 8, 8), (256, 2, 1, 16)])
def test_plan_head_mapping(lib, Hq, Hkv, hg, ncw):
    rc, p = plan(lib, 4, Hq, Hkv)
    assert rc == 0
    assert p.heads_per_row == hg and p.consumer_warps == ncw
    assert p.threads == 32 * (ncw + 1)
    assert 2 <= p.stages <= 8 and p.smem_bytes <= 227 * 1024


def test_plan_rejects_bad_shapes(lib):
    assert plan(lib, 4, 30, 8)[0] == -1   # Hq % Hkv != 0
    assert plan(lib, 4, 0, 8)[0] == -1
    assert plan(lib, 4, 129 * 8, 8)[0] == -2  # group of 129 heads
    assert plan(lib, 4, 32, 8, ns=513)[0] == -1


def test_plan_fixed_workspace_matches_reference_layout(lib):
    # [B, Hq, ns, 128] + [B, Hq, ns] x 2, fp32 (python/gqa_decode_ext.cpp:106-109)
    rc, p = plan(lib, 32, 32, 8, ns=8)
    states = 32 * 32 * 8
    assert p.workspace_bytes == states * 128 * 4 + 2 * align256(states * 4)
    assert p.grid == min(148, 32 * 8)
    rc, p = plan(lib, 32, 32, 8, ns=1)
    assert p.workspace_bytes == 0 and p.grid == 32


def test_pick_splits(lib):
    # rep shape: 32 rows; the chosen count fills the waves it uses to >= 90 %.
    ns = lib.gqa_decode_pick_splits(32, 32, 8, 8192, 148)
    assert 1 < ns <= 512
    tasks = 32 * ns
    waves = -(-tasks // 148)
    assert tasks / (waves * 148) >= 0.9
    # one long request: many splits
    assert lib.gqa_decode_pick_splits(1, 32, 8, 262144, 148) >= 100
    # a batch that already fills the GPU several times: no split
    assert lib.gqa_decode_pick_splits(4096, 32, 8, 512, 148) == 1
    assert lib.gqa_decode_pick_splits(0, 32, 8, 512, 148) == 1


def test_declares_every_header(lib):
    names = declared_functions()
    for expected in ("gqa_decode_launch", "mla_decode_launch", "mla_decode_sparse_launch",
                     "dsa_indexer_launch", "dsa_topk_launch", "dsa_gather_launch",
                     "dsa_decode_get_status"):
        assert expected in names


def test_mla_splits_and_workspace(lib):
    lib.mla_decode_pick_splits.argtypes = [ctypes.c_int] * 5
    lib.mla_decode_pick_splits.restype = ctypes.c_int
    lib.mla_decode_workspace_bytes.argtypes = [ctypes.c_int] * 4
    lib.mla_decode_workspace_bytes.restype = ctypes.c_size_t
    # 128-row query groups run the persistent kernel: one split, and a
    # workspace (partial states, unit layout) whatever num_splits is
    assert lib.mla_decode_pick_splits(128, 1, 128, 128, 148) == 1
    assert lib.mla_decode_pick_splits(4, 2, 64, 4096, 148) == 1  # s_q * h_q = 128
    for ns in (1, 4):
        assert lib.mla_decode_workspace_bytes(128, 1, 128, ns) > 0
        assert lib.mla_decode_workspace_bytes(4, 2, 64, ns) > 0
    # smaller groups: split partial states only for num_splits > 1
    assert lib.mla_decode_workspace_bytes(128, 1, 16, 1) == 0
    assert lib.mla_decode_workspace_bytes(128, 1, 16, 4) >= 128 * 16 * 4 * 512 * 4
    # one long request with few heads is split; bad shapes fall back to 1
    assert lib.mla_decode_pick_splits(1, 1, 16, 4096, 148) > 1
    assert lib.mla_decode_pick_splits(0, 1, 16, 4096, 148) == 1
    assert lib.mla_decode_workspace_bytes(0, 1, 128, 1) == 0


def test_balanced_workspace_for_huge_batches_and_grid_cap(lib):
    # the layout scales with rows; the grid is capped at 2048 CTAs
    rc, p = plan(lib, 16384, 32, 8)
    assert rc == 0 and p.workspace_bytes == balanced_bytes(148, 16384, rows=16384, qhr=32)
    rc, p = plan(lib, 64, 32, 1, sms=148, per_sm=20)
    assert rc == 0 and p.grid == 2048


def test_selftests_reject_bad_arguments_before_any_device_call(lib):
    # argument checks come first, so these return without a GPU
    P, PP, I, Z = ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_size_t
    f = lib.gqa_decode_selftest_kvshard_emulated
    f.argtypes = [P, P, P, PP, PP, PP] + [I] * 7 + [ctypes.c_float, P, Z, P, Z, P]
    f.restype = I
    arr = (ctypes.c_void_p * 1)(None)
    for world in (1, 9):  # one rank is no exchange; more than 8 peers is unsupported
        assert f(None, None, None, arr, arr, arr, world, 1, 32, 8, 16, 4, 0, 1.0, None, 0,
                 None, 0, None) == 1  # cudaErrorInvalidValue
    g = lib.gqa_decode_selftest_kvshard_emulated_bytes
    g.argtypes = [I] * 4 + [ctypes.POINTER(Z)]
    g.restype = Z
    assert g(1, 32, 8, 1, None) == 0 and g(1, 33, 8, 2, None) == 0 and g(0, 32, 8, 2, None) == 0
    h = lib.gqa_decode_selftest_exchange_timeout
    h.argtypes = [P] * 6 + [I] * 5 + [ctypes.c_float, I, P, Z, P, Z, P]
    h.restype = I
    for wait_us in (0, 1000001):
        assert h(None, None, None, None, None, None, 1, 32, 8, 16, 4, 1.0, wait_us, None, 0,
                 None, 0, None) == 1
