"""Loader for the reference golden vectors in ``tests/golden/reference_cases.npz``.

The vectors were produced by ``tests/golden/make_golden.py``, which runs the
reference's own Triton kernels (npu_flash_attention.py) on the CPU.
"""
import json
import os

import numpy as np
import torch

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                    "reference_cases.npz")
DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def _load_tensor(arr: np.ndarray, dtype: str) -> torch.Tensor:
    if arr.dtype == np.uint16:
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(arr.copy())


def load_cases():
    z = np.load(PATH)
    metas = json.loads(bytes(z["__meta__"]).decode())
    cases = []
    for meta in metas:
        name = meta["name"]
        rec = {}
        for key in z.files:
            if key.startswith(name + "/"):
                field = key.split("/", 1)[1]
                if field in ("lse", "alibi_slope"):
                    rec[field] = torch.from_numpy(z[key].copy())
                else:
                    rec[field] = _load_tensor(z[key], meta["dtype"])
        cases.append((meta, rec))
    return cases
