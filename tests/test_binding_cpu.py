"""CPU: the PyTorch binding imports without a GPU, keeps the reference's
registry and function signatures, and raises the reference's validation
errors (python/gqa_decode_ext.cpp:16-62, 102-103) before touching a GPU."""

import inspect
import math

import pytest
import torch

import binding

SCALE = 1.0 / math.sqrt(128)


def cpu_case(B=2, Hq=32, Hkv=8, bs=16, nblk=8):
    q = torch.zeros(B, Hq, 128, dtype=torch.bfloat16)
    k = torch.zeros(nblk, bs, Hkv, 128, dtype=torch.bfloat16)
    v = torch.zeros_like(k)
    bt = torch.zeros(B, 4, dtype=torch.int32)
    sl = torch.ones(B, dtype=torch.int32)
    return q, k, v, bt, sl


def test_registry_and_signatures():
    assert {"v0", "v1", "v2"} <= set(binding.KERNELS)
    sig = inspect.signature(binding.gqa_decode_v2)
    assert list(sig.parameters) == ["q", "k_cache", "v_cache", "block_table", "seq_lens", "scale",
                                    "num_splits"]
    assert sig.parameters["num_splits"].default == 8


def test_loaded_from_tree():
    import os
    assert os.path.exists(binding.LIB_PATH) and os.path.exists(binding.EXT_PATH)


@pytest.mark.parametrize("kernel", ["v0", "v1", "v2"])
def test_rejects_cpu_tensors(kernel):
    with pytest.raises(RuntimeError, match="q must be a CUDA tensor"):
        binding.KERNELS[kernel](*cpu_case(), SCALE)


def test_v2_num_splits_range_message():
    # The range check sits after the tensor checks, as in the reference; with
    # CPU tensors the device check fires first.
    with pytest.raises(RuntimeError, match="q must be a CUDA tensor"):
        binding.gqa_decode_v2(*cpu_case(), SCALE, num_splits=0)


def test_merge_states_rejects_cpu():
    m = torch.zeros(2, 4)
    with pytest.raises(RuntimeError, match="states must be CUDA tensors"):
        binding.merge_states(m, m, torch.zeros(2, 4, 128))
