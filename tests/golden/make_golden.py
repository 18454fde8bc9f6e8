"""Generates the golden fixtures of tests/golden/ (run in the build container).

Inputs are the reference's own decode-test tensors: `cached_randn` of
tests/inductor/utils_inductor.py:27-50 with the shapes and differentiation tags
of the `mha_decode` / `gqa_decode` param sets (tests/inductor/
test_inductor_ops.py:2651-2678) and of test_index_copy_inplace_{prefill,decode}
(5688-5740).  When a checkout of the reference is given (``--reference DIR``
or the environment variable TORCH_SPYRE_REFERENCE, the root of a torch-spyre
tree) its `cached_randn` is imported (the spyre device name is registered
first so the module imports without the Spyre runtime) and checked against
this repo's `seeded_randn`; otherwise `seeded_randn` alone is used.

Usage: python tests/golden/make_golden.py [--reference DIR]

Outputs are what the reference's harness treats as the truth: the test
function run eagerly on CPU tensors (compare_with_cpu,
tests/inductor/utils_inductor.py:620-703).  The reference's decode param sets
hand SDPA [B, S, H, D] tensors without the transpose(1, 2) its prefill sets
apply (and mark the cases expect_fail); the fixtures apply the transpose, so
q is [B, H, 1, D] and k/v are [B, Hkv, 257, D].

The rotary embedding fixtures evaluate the reference's rope dataflow
(tests/inductor/test_inductor_ops.py:5447-5456: view the row as two halves,
multiply by freqs broadcast over the output half, sum over the input half,
flatten) on its own param sets (2840-2858) with CPU fp16 tensors.

Writes sdpa_decode_golden.npz, index_copy_golden.json and rope_golden.json /
rope_golden.npz.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from torch_spyre_b200.workloads import seeded_randn  # noqa: E402

def reference_tests_dir():
    """tests/inductor of the reference checkout named on the command line or in
    TORCH_SPYRE_REFERENCE (None if neither names an existing tree)."""
    import argparse
    import os

    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TORCH_SPYRE_REFERENCE"),
                    help="root of a torch-spyre checkout whose cached_randn pins the inputs")
    root = ap.parse_args().reference
    if not root:
        return None
    d = Path(root) / "tests" / "inductor"
    return d if d.exists() else None


def reference_randn():
    REF_TESTS = reference_tests_dir()
    if REF_TESTS is None:
        return None
    try:
        torch.utils.rename_privateuse1_backend("spyre")
    except RuntimeError:
        pass
    sys.path.insert(0, str(REF_TESTS))
    import utils_inductor  # noqa: E402

    return utils_inductor.cached_randn


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.int16).numpy().tobytes()).hexdigest()


def main():
    ref = reference_randn()
    pinned_by_reference = ref is not None

    def randn(shape, differentiation=None):
        ours = seeded_randn(shape, differentiation=differentiation, dtype=torch.float16)
        if ref is not None:
            theirs = ref(shape, differentiation=differentiation, dtype=torch.float16)
            assert torch.equal(ours, theirs), "seeded_randn diverges from the reference cached_randn"
        return ours

    cases = {"mha_decode": 32, "gqa_decode": 8}
    arrays = {}
    meta = {"pinned_by_reference_cached_randn": pinned_by_reference, "torch": torch.__version__}
    for name, hkv in cases.items():
        q = randn((2, 1, 32, 128), 1).transpose(1, 2)        # [2, 32, 1, 128]
        k = randn((2, 257, hkv, 128), 2).transpose(1, 2)     # [2, Hkv, 257, 128]
        v = randn((2, 257, hkv, 128), 3).transpose(1, 2)
        gqa = hkv != 32
        out_native = F.scaled_dot_product_attention(q, k, v, enable_gqa=gqa)
        out_fp32 = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), enable_gqa=gqa)
        s = (q.float() @ k.float().repeat_interleave(32 // hkv, 1).transpose(-2, -1)) / np.sqrt(128)
        arrays[f"{name}_out_native"] = out_native.numpy()
        arrays[f"{name}_out_fp32"] = out_fp32.numpy()
        arrays[f"{name}_lse"] = torch.logsumexp(s[:, :, 0], dim=-1).numpy()
        meta[name] = {"sha_q": sha(q), "sha_k": sha(k), "sha_v": sha(v), "num_kv_heads": hkv}
    np.savez_compressed(HERE / "sdpa_decode_golden.npz", **arrays)

    # index_copy_ KV append, prefill then decode (test_inductor_ops.py:5688-5740)
    cache = randn((1, 8, 2048, 128))
    src_prefill = randn((1, 8, 14, 128), "prefill")
    src_decode = randn((1, 8, 1, 128), "decode")
    after_prefill = cache.clone().index_copy_(2, torch.arange(14), src_prefill)
    after_decode = cache.clone().index_copy_(2, torch.tensor([14]), src_decode)
    ic = {
        "pinned_by_reference_cached_randn": pinned_by_reference,
        "sha_cache": sha(cache),
        "sha_after_prefill": sha(after_prefill),
        "sha_after_decode": sha(after_decode),
    }
    (HERE / "index_copy_golden.json").write_text(json.dumps(ic, indent=1) + "\n")

    # rotary embedding (test_inductor_ops.py:2840-2858 inputs, 5447-5456 dataflow)
    rope_meta, rope_arrays = {"pinned_by_reference_cached_randn": pinned_by_reference}, {}
    for name, qshape, fshape in [("prefill_bs1", (1, 256, 4096), (1, 256, 2, 2, 64)),
                                 ("prefill", (2, 256, 4096), (1, 256, 2, 2, 64)),
                                 ("decode_bs1", (1, 1, 4096), (1, 1, 2, 2, 64)),
                                 ("decode", (2, 1, 4096), (1, 1, 2, 2, 64))]:
        q, freqs = randn(qshape), randn(fshape)
        B, S, E = q.shape
        D = freqs.shape[-1] * 2
        halves = q.view(B, S, E // D, 2, D // 2).unsqueeze(-3)      # [B, S, H, 1, 2, D/2]
        out = (freqs[:, :, None] * halves).sum(4, keepdim=True).flatten(3)
        rope_meta[name] = {"q_shape": list(qshape), "freqs_shape": list(fshape), "sha_q": sha(q),
                           "sha_freqs": sha(freqs), "sha_out": sha(out), "out_shape": list(out.shape)}
        if S == 1:
            rope_arrays[f"{name}_out"] = out.numpy()
    (HERE / "rope_golden.json").write_text(json.dumps(rope_meta, indent=1) + "\n")
    np.savez_compressed(HERE / "rope_golden.npz", **rope_arrays)
    (HERE / "sdpa_decode_golden.json").write_text(json.dumps(meta, indent=1) + "\n")
    print("wrote fixtures; pinned by reference cached_randn:", pinned_by_reference)


if __name__ == "__main__":
    main()
