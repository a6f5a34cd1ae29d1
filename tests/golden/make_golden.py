"""Generate the golden attention fixtures from the reference's own oracle.

Runs ``attention_reference`` of the reference project
(``flash_attention/reference.py:9-61``) on seeded fp16 inputs, called with
the fp32 upcast of those inputs so the stored output is the reference's fp32
result, and writes ``tests/golden/attention_golden.npz``.

This script needs the reference checkout (pass its path); the fixtures it
writes are committed so the tests do not.

    python tests/golden/make_golden.py REFERENCE_ROOT
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# (name, B, H, Nq, Nk, D, causal, scale, stress)
CASES = [
    ("b1h1n1d16", 1, 1, 1, 1, 16, False, None, False),
    ("b1h1n1d16_causal", 1, 1, 1, 1, 16, True, None, False),
    ("b1h2n17d32", 1, 2, 17, 17, 32, False, None, False),
    ("b1h2n17d32_causal", 1, 2, 17, 17, 32, True, None, False),
    ("b2h4n64d64", 2, 4, 64, 64, 64, False, None, False),
    ("b2h4n64d64_causal", 2, 4, 64, 64, 64, True, None, False),
    ("b1h2n128d64", 1, 2, 128, 128, 64, False, None, False),
    ("b1h2n128d64_causal", 1, 2, 128, 128, 64, True, None, False),
    ("b1h1n384d64_causal", 1, 1, 384, 384, 64, True, None, False),
    ("b1h1n200d64", 1, 1, 200, 200, 64, False, None, False),
    ("b1h1n200d64_causal", 1, 1, 200, 200, 64, True, None, False),
    ("b1h1q100k300d64", 1, 1, 100, 300, 64, False, None, False),
    ("b1h1q100k300d64_causal", 1, 1, 100, 300, 64, True, None, False),
    ("b1h1q300k100d64_causal", 1, 1, 300, 100, 64, True, None, False),
    ("b1h2n128d64_scale0.3", 1, 2, 128, 128, 64, False, 0.3, False),
    ("b1h1n256d64_stress", 1, 1, 256, 256, 64, False, None, True),
    ("b1h1n256d64_stress_causal", 1, 1, 256, 256, 64, True, None, True),
]


def load_reference(root: Path):
    spec = importlib.util.spec_from_file_location(
        "reference_oracle", root / "flash_attention" / "reference.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.attention_reference


def make_case(seed: int, b: int, h: int, nq: int, nk: int, d: int, stress: bool):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, nq, d, generator=g)
    k = torch.randn(b, h, nk, d, generator=g)
    v = torch.randn(b, h, nk, d, generator=g)
    if stress:
        q, k = q * 8, k * 8
        n_out = max(1, round(0.01 * nk))
        for bi in range(b):
            for hi in range(h):
                rows = torch.randperm(nk, generator=g)[:n_out]
                sign = torch.randint(0, 2, (n_out, d), generator=g) * 2 - 1
                k[bi, hi, rows] = 30.0 * sign.float()
    return q.half(), k.half(), v.half()


def main(root: Path) -> None:
    attention_reference = load_reference(root)
    out = {}
    for i, (name, b, h, nq, nk, d, causal, scale, stress) in enumerate(CASES):
        q, k, v = make_case(1000 + i, b, h, nq, nk, d, stress)
        ref = attention_reference(q.float(), k.float(), v.float(), causal=causal, scale=scale)
        out[f"{name}/q"] = q.numpy()
        out[f"{name}/k"] = k.numpy()
        out[f"{name}/v"] = v.numpy()
        out[f"{name}/out"] = ref.numpy().astype(np.float32)
        out[f"{name}/meta"] = np.array([b, h, nq, nk, d, int(causal),
                                        -1.0 if scale is None else scale], dtype=np.float64)
    np.savez_compressed(HERE / "attention_golden.npz", **out)
    print(f"wrote {len(CASES)} cases to {HERE / 'attention_golden.npz'}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(Path(sys.argv[1]))
