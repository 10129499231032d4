"""Regenerate the Task 02 golden fixtures from the reference implementation itself.

Runs dsa_topk_page_table_transform of sinpeyw/flagos-kernelgen-72h-shanghai-2026
(src/task02_dsa_topk_page_table_transform.py) on CPU tensors under Triton's
interpreter (TRITON_INTERPRET=1). On CPU tensors its backend tag holds no
vendor name, so its routing falls through to 'nvidia' (:32-51) and picks the
NVIDIA kernels of each shape. Stores out_blocks and out_pages per case as
tests/golden/topk_<case>.npz with a digest of the inputs.

One shim, in the interpreter only: Triton 3.6's interpreter builds the
all-ones constant of `~x` as np.full(1, -1, dtype=uint32), which numpy 2
rejects; here it is built as np.array([-1]).astype(uint32) (the same bits).

Usage (needs the reference checkout; not run by the tests):
    python tests/golden/make_golden_topk.py /path/to/src/task02_dsa_topk_page_table_transform.py
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
from triton.runtime import interpreter as _interp  # noqa: E402

from topk_cases import TOPK_CASES, topk_case_inputs, topk_input_digest  # noqa: E402

_orig_all_ones = _interp.InterpreterBuilder.get_all_ones_value


def _all_ones(self, type):
    np_type = _interp._get_np_dtype(type)
    if "int" in np_type.name:
        return _interp.TensorHandle(np.array([-1]).astype(np_type), type.scalar)
    return _orig_all_ones(self, type)


_interp.InterpreterBuilder.get_all_ones_value = _all_ones


def load_reference(path: str):
    spec = importlib.util.spec_from_file_location("reference_task02", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(ref_path: str, only: list[str]) -> None:
    ref = load_reference(ref_path)
    for name in TOPK_CASES:
        if only and name not in only:
            continue
        w, scores, pt, q_pos, kv = topk_case_inputs(name)
        assert ref._backend_name(scores) == "nvidia"
        ob = torch.empty(w.B, w.H, w.Q, w.top_k, dtype=torch.int32)
        op = torch.empty(w.B, w.H, w.Q, w.top_k, dtype=torch.int32)
        t0 = time.time()
        ref.dsa_topk_page_table_transform(scores, pt, q_pos, kv, ob, op, w.block_size, w.top_k)
        np.savez_compressed(HERE / f"topk_{name}.npz", out_blocks=ob.numpy(),
                            out_pages=op.numpy(),
                            digest=np.array(topk_input_digest(scores, pt, q_pos, kv)),
                            route=np.array(TOPK_CASES[name][1]))
        print(f"{name}: {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2:])
