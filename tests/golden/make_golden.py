"""Regenerate the golden fixtures from the reference implementation itself.

Runs fused_add_rmsnorm_group_quant of sinpeyw/flagos-kernelgen-72h-shanghai-2026
(src/task01_fused_add_rmsnorm_group_quant.py) on CPU tensors under Triton's
interpreter (TRITON_INTERPRET=1), with its backend tag fixed to an NVIDIA
B200 so the NVIDIA routing (:1772-1817, :1548-1728) picks the kernel, and
stores x_q (int8) and x_scale (fp32) per case as tests/golden/<case>.npz.

The interpreter truncates fp32 -> bf16/fp16 stores, unlike a GPU (which
rounds to nearest even), so residual_out and norm_out are NOT stored: their
bit-exact oracle is the RNE cast of the fp32 sum.

Usage (needs the reference checkout; not run by the tests):
    python tests/golden/make_golden.py /path/to/src/task01_fused_add_rmsnorm_group_quant.py
"""
from __future__ import annotations

import importlib.util
import os
import sys
import time
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"
HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from cases import CASES, case_inputs, input_digest, stored_rows  # noqa: E402


def load_reference(path: str):
    spec = importlib.util.spec_from_file_location("reference_task01", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod._backend_tag = lambda t: "cuda nvidia b200"
    return mod


def main(ref_path: str, only: list[str]) -> None:
    ref = load_reference(ref_path)
    for name in CASES:
        if only and name not in only:
            continue
        w, x, r, g = case_inputs(name)
        M, D, G = w.M, w.D, w.group_size
        ro = torch.empty_like(x)
        no = torch.empty(M, D, dtype=torch.bfloat16)
        q = torch.empty(M, D, dtype=torch.int8)
        s = torch.empty(M, D // G, dtype=torch.float32)
        t0 = time.time()
        ref.fused_add_rmsnorm_group_quant(x, r, g, ro, no, q, s, w.eps, G)
        np.savez_compressed(HERE / f"{name}.npz", q=stored_rows(name, q).numpy(),
                            scale=stored_rows(name, s).numpy(),
                            digest=np.array(input_digest(x, r, g)),
                            kernel=np.array(CASES[name][2]))
        print(f"{name}: {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2:])
