"""Generate tests/golden/golden.npz from the reference's own fp32 oracle.

Runs the UNMODIFIED python/reference.py of yuqiz7/mla-decode-kernels
(attention_ref, reference.py:21-40) on seeded inputs built by
mla-decode-kernels_b200/python/cases.py and stores, per case, the reference
output and a SHA-256 of the inputs.  The tests rebuild the inputs with the
same recipe, check the hash (so a changed RNG is caught, not mistaken for a
parity failure) and compare the CPU oracle against the stored output.

Usage (needs the reference checkout; the fixtures then travel without it):
    python tests/golden/make_golden.py --reference /path/to/mla-decode-kernels
"""

import argparse
import hashlib
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "mla-decode-kernels_b200", "python"))
sys.path.insert(0, os.path.join(REPO, "oracle"))

import cases  # noqa: E402


def input_digest(case):
    h = hashlib.sha256()
    for t in case:
        t = t.contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        h.update(t.numpy().tobytes())
    return h.hexdigest()


def golden_cases():
    """name -> (builder, description).  Small enough for pure CPU."""
    out = {}
    out["config1"] = (lambda: cases.config1(device="cpu"), "BASELINE config 1")
    for name in ["a_base", "b_long", "c_len1", "d_exact_blocks", "e_partial_blocks", "f_bs64",
                 "g_hq64", "i_8k"]:
        out["ref_" + name] = (lambda n=name: cases.ref_case(n, seed=0), "reference test case " + name)
    out["peaked_k8"] = (
        lambda: cases.make_case([700, 129], 32, 8, 16, seed=11, k_scale=8.0),
        "K x8 peaked softmax")
    out["large_logits_q50"] = (
        lambda: cases.make_case([100, 257, 512, 33], 32, 8, 16, seed=12, value_scale=0.5,
                                k_scale=1.0),
        "q x50 (applied by the test) large logits")
    out["ragged_mini"] = (
        lambda: cases.make_case(cases.config4_seq_lens(seed=1, B=6), 32, 8, 16, seed=13,
                                pool_factor=1.0 / 0.9),
        "config-4 recipe, 6 requests")
    out["long_mini_bs64"] = (
        lambda: cases.make_case([16384], 32, 8, 64, seed=14, pool_factor=1.0),
        "config-5 recipe, 16K tokens")
    out["group16"] = (
        lambda: cases.make_case([300, 45], 64, 4, 16, seed=15), "Hq/Hkv = 16")
    out["mha_group1"] = (
        lambda: cases.make_case([77, 300], 8, 8, 16, seed=16), "Hq == Hkv")
    out["empty_request"] = (
        lambda: cases.make_case([50, 0, 17], 32, 8, 16, seed=17), "a request with seq_len 0")
    return out


def q_transform(name, q):
    if name == "large_logits_q50":
        return (q.float() * 50.0).to(torch.bfloat16)
    return q


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None,
                    help="reference checkout (default: GQA_REFERENCE_DIR, else the "
                         "reference_path recorded in BASELINE.json)")
    ap.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    args = ap.parse_args()
    if args.reference is None:
        import oracle

        args.reference = oracle.reference_checkout()
    if args.reference is None:
        raise SystemExit("make_golden.py needs the reference checkout: pass --reference or set "
                         "GQA_REFERENCE_DIR")
    sys.path.insert(0, os.path.join(args.reference, "python"))
    from reference import attention_ref  # the reference's own oracle

    torch.set_num_threads(os.cpu_count())
    scale = 1.0 / math.sqrt(128)
    arrays = {}
    for name, (builder, desc) in golden_cases().items():
        q, k, v, bt, sl = builder()
        q = q_transform(name, q)
        case = (q, k, v, bt, sl)
        out = attention_ref(q, k, v, bt, sl, scale)
        arrays[name + "/out"] = out.numpy().astype(np.float32)
        arrays[name + "/digest"] = np.array(input_digest(case))
        print(f"{name:20s} {desc:40s} out {tuple(out.shape)} digest {input_digest(case)[:16]}")
    np.savez_compressed(args.out, **arrays)
    print("wrote", args.out, os.path.getsize(args.out), "bytes")


if __name__ == "__main__":
    main()
