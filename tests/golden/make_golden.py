"""Generate the golden fixtures in tests/golden/ from the REFERENCE's own naive
kernel (methodology/checkpoints/kernel_naive.cu compiled for CPU by
oracle/build_ref.py).  Run in the development container, where the
reference tree is mounted:

    python tests/golden/make_golden.py

Each fixture stores the reference's outputs, checksums of the inputs and,
for the one-page case, the complete inputs.  The other cases (and benchmark
config 1, whose 8 MiB pool is too large to commit) are rebuilt from the
seeded generators in tests/golden/cases.py; the checksums prove the rebuilt
inputs are the ones the reference saw.
"""
from __future__ import annotations

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.build_ref import build_ref, load_ref  # noqa: E402
from tests.golden.cases import CASES, checksum, INPUT_KEYS  # noqa: E402


def main():
    build_ref()
    ref = load_ref()
    if ref is None:
        raise SystemExit("reference module unavailable")
    for name, make in CASES.items():
        w = make()
        out = torch.empty((w.num_tokens, 16, 512), dtype=torch.bfloat16)
        lse = torch.empty((w.num_tokens, 16), dtype=torch.float32)
        ref.launch_sparse_attention_c(*w.args(), out, lse)
        rec = {"case": name, "sm_scale": w.sm_scale,
               "checksums": {k: checksum(getattr(w, k)) for k in INPUT_KEYS},
               "output": out, "lse": lse, "generator": "reference kernel_naive.cu (CPU build)"}
        if w.ckv_cache.numel() <= 64 * 512:
            rec["inputs"] = {k: getattr(w, k) for k in INPUT_KEYS}
        torch.save(rec, os.path.join(HERE, f"{name}.pt"))
        print(name, w.num_tokens, w.num_pages)


if __name__ == "__main__":
    main()
