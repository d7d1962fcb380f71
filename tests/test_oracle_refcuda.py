"""The oracle against outputs of the reference's own CUDA extension.

tests/golden/reference_cuda.npz holds pack + score outputs of the reference's
csrc/popkv_ext.{cpp,cu}, compiled unmodified (with its -O3 --use_fast_math flags)
and run on a B200 by tests/golden/make_golden_refcuda.py.  The oracle restates the
kernel with IEEE division and a correctly rounded 1/sqrt(D); fast-math division
differs from it in the last bits, so:
  * sign and magnitude bitmasks: identical (pure fp32 compares);
  * fp16 representatives: identical except a small fraction, each off by at most
    a few fp16 ulps (cancellation in high - low after the approximate division);
  * scores: within 1e-3 relative of the score scale (the north star's tolerance).
"""
from pathlib import Path

import numpy as np
import pytest

import popkv_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_cuda.npz"
NAMES = sorted({k.split("/")[0] for k in np.load(GOLDEN).files})


@pytest.fixture(scope="module")
def ref():
    return np.load(GOLDEN)


@pytest.mark.parametrize("name", NAMES)
def test_oracle_pack_matches_reference_kernel(ref, name):
    keys = ref[f"{name}/keys"]
    sign, mag, low, delta = O.pack_keys(keys)
    np.testing.assert_array_equal(sign, ref[f"{name}/k_sign"])
    np.testing.assert_array_equal(mag, ref[f"{name}/k_mag"])
    for ours, theirs in ((low, ref[f"{name}/low"]), (delta, ref[f"{name}/delta"])):
        a = O.f16_bits_to_float(ours).astype(np.float64)
        b = O.f16_bits_to_float(theirs).astype(np.float64)
        differ = ours != theirs
        assert differ.mean() < 2e-3, differ.mean()
        scale = np.abs(b).max()
        assert np.all(np.abs(a - b) <= 2 ** -9 * np.maximum(np.abs(b), 2 ** -6 * scale))


@pytest.mark.parametrize("name", NAMES)
def test_oracle_scores_match_reference_kernel(ref, name):
    keys, queries = ref[f"{name}/keys"], ref[f"{name}/queries"]
    h2k = ref[f"{name}/head_to_kv"]
    packed = O.pack_keys(keys)
    got = O.score(queries, packed, head_to_kv=h2k, tokens=keys.shape[1])
    want = ref[f"{name}/scores"]
    scale = np.abs(want).max()
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-3 * scale)
    # Scoring the reference kernel's own packed cache: only the scale differs
    # (fast-math rsqrtf vs the correctly rounded 1/sqrt(D)).
    theirs = tuple(ref[f"{name}/{k}"] for k in ("k_sign", "k_mag", "low", "delta"))
    again = O.score(queries, theirs, head_to_kv=h2k, tokens=keys.shape[1])
    np.testing.assert_allclose(again, want, rtol=2e-6, atol=1e-6 * scale)
