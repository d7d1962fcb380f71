"""The new kernels against the reference's own CUDA extension, run side by side.

oracle/_ref holds csrc/popkv_ext.{cpp,cu} of the reference compiled unmodified
with its -O3 --use_fast_math flags (oracle/build_ref.py).  Bitmasks must match
bit for bit; with reference division the fp16 representatives and scores match
too; in the default IEEE mode representatives may differ by one fp16 ulp where
the reference's approximate division rounds the other way.
"""
import numpy as np
import pytest
import torch

import build_ref
import popkv_cuda as pk
from conftest import packed_numpy, synthetic_keys

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def ref():
    ext = build_ref.load()
    if ext is None:
        pytest.skip("reference extension not built in oracle/_ref")
    return ext


def _pair(ref, kvh, qh, tokens, dim, dtype, seed, flags):
    k = synthetic_keys(kvh, tokens, dim, seed=seed, dtype=dtype).to(DEV)
    q = synthetic_keys(1, qh, dim, seed=seed + 1, dtype=dtype).to(DEV)
    h2k = (torch.arange(qh) // (qh // kvh)).to(DEV)
    theirs = ref.pack(k, tokens)
    ours = pk.pack_keys(k, token_capacity=tokens, flags=flags)
    s_theirs = ref.score(q, *theirs, h2k, tokens)
    s_ours = pk.score(q, ours, head_to_kv=h2k, tokens=tokens, flags=flags)
    torch.cuda.synchronize()
    return packed_numpy(ours), packed_numpy(theirs), s_ours.cpu().numpy(), s_theirs.cpu().numpy()


CASES = [(8, 32, 32768, 128, torch.bfloat16), (2, 8, 37, 64, torch.bfloat16),
         (2, 8, 1000, 96, torch.float32), (1, 4, 45, 128, torch.float16)]


@pytest.mark.parametrize("case", CASES)
def test_bitmasks_identical_and_scores_close(ref, case):
    ours, theirs, s_ours, s_theirs = _pair(ref, *case, seed=case[2], flags=0)
    np.testing.assert_array_equal(ours[0], theirs[0])
    np.testing.assert_array_equal(ours[1], theirs[1])
    for a, b in ((ours[2], theirs[2]), (ours[3], theirs[3])):
        fa = a.view(np.float16).astype(np.float32)
        fb = b.view(np.float16).astype(np.float32)
        # IEEE vs approximate division: a few fp32 ulps before the fp16 rounding,
        # which can move delta = high - low by more than one fp16 ulp when high ~ low.
        assert (a != b).mean() < 1e-3
        assert (np.abs(fa - fb) <= 2.0 ** -9 * np.maximum(1.0, np.abs(fb))).all()
    np.testing.assert_allclose(s_ours, s_theirs, rtol=1e-3, atol=1e-3 * np.abs(s_theirs).max())


@pytest.mark.parametrize("case", CASES)
def test_reference_division_mode_is_bit_identical(ref, case):
    ours, theirs, s_ours, s_theirs = _pair(ref, *case, seed=case[2] + 5, flags=pk.REFERENCE_DIVISION)
    for a, b in zip(ours, theirs):
        np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(s_ours, s_theirs)
