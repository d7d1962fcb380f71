"""Record outputs of the reference's own CUDA extension as fixtures (run on a GPU).

Usage:  python tests/golden/make_golden_refcuda.py <out.npz>

Loads oracle/_ref/popkv_ext_ref*.so (the reference's csrc/popkv_ext.{cpp,cu},
compiled unmodified with its own -O3 --use_fast_math flags by
oracle/build_ref.py) and records pack + score for seeded inputs.  The committed
file tests/golden/reference_cuda.npz lets the CPU tests pin the oracle against
the reference kernels without a GPU.
"""
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
import build_ref  # noqa: E402

CASES = [  # name, seed, kvh, qh, tokens, dim, dtype
    ("bf16_d128", 1, 2, 8, 200, 128, torch.bfloat16),
    ("bf16_d64_ref_test", 11, 2, 8, 37, 64, torch.bfloat16),
    ("fp32_d96", 2, 2, 4, 70, 96, torch.float32),
    ("fp16_d128_partial", 3, 1, 4, 45, 128, torch.float16),
]


def main(out_path: str) -> None:
    ext = build_ref.load()
    if ext is None:
        raise SystemExit("reference extension not built (oracle/build_ref.py)")
    out = {}
    for name, seed, kvh, qh, tokens, dim, dtype in CASES:
        g = torch.Generator().manual_seed(seed)
        keys = torch.randn(kvh, tokens, dim, generator=g)
        for h in range(kvh):
            keys[h, :, torch.randperm(dim, generator=g)[:4]] *= 8.0
        queries = torch.randn(1, qh, dim, generator=g) * 2
        keys, queries = keys.to(dtype), queries.to(dtype)
        mapping = torch.arange(qh) // (qh // kvh)
        packed = ext.pack(keys.cuda().contiguous(), tokens)
        scores = ext.score(queries.cuda().contiguous(), *packed, mapping.cuda(), tokens)
        torch.cuda.synchronize()
        out[f"{name}/keys"] = keys.float().numpy()
        out[f"{name}/queries"] = queries.float().numpy()
        out[f"{name}/head_to_kv"] = mapping.numpy()
        out[f"{name}/k_sign"] = packed[0].cpu().numpy()
        out[f"{name}/k_mag"] = packed[1].cpu().numpy()
        out[f"{name}/low"] = packed[2].cpu().view(torch.int16).numpy().view(np.uint16)
        out[f"{name}/delta"] = packed[3].cpu().view(torch.int16).numpy().view(np.uint16)
        out[f"{name}/scores"] = scores.cpu().numpy()
    np.savez_compressed(out_path, **out)
    print("wrote", out_path, len(out), "arrays")


if __name__ == "__main__":
    main(sys.argv[1])
