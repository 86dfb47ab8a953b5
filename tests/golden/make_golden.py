"""Generate golden vectors by running the REFERENCE's own kernels on the CPU.

The reference (dropletzhu/npu-flex-att, ``npu_flash_attention.py``) is Triton
DSL written for Ascend NPUs. Its kernels run unchanged under Triton's CPU
interpreter (``TRITON_INTERPRET=1``) once three Ascend-only names are supplied:

* ``import torch_npu``                     -> an empty stand-in module;
* ``triton.language.extra.ascend.libdevice`` -> an empty stand-in module
  (imported at npu_flash_attention.py:10-13 but never used);
* ``tl.tanh`` (Ascend extension used for soft-cap at :106, :376, :492, :536)
  -> ``tanh(x) = sign(x)·(1 − e^{−2|x|}) / (1 + e^{−2|x|})``, written here from
  the definition of tanh.

The launch keyword ``multibuffer=True`` (Ascend-only) is ignored by the
interpreter. The interpreter computes through numpy, which has no bfloat16:
bf16 launches return garbage there. bf16 cases therefore run the reference
kernels at fp32 on the exact bf16-valued inputs and carry the flag
``ref_computed_in_fp32``; their outputs are stored as float32. Everything else -- tiling, online softmax, masks, GQA mapping,
the backward kernels and host-side Δ / GQA sum -- is the reference's own code.

Run this in a container that has the reference checked out (it is NOT run by
the tests, and nothing on the GPU box reads the reference):

    python tests/golden/make_golden.py /path/to/reference  [out.npz]

(or with the checkout's path in the environment variable NPU_FLEX_ATT_REFERENCE).

Inputs are drawn with ``torch.manual_seed`` on the CPU in fp32 and cast, so
the stored inputs are exact. Every case stores its inputs, the reference's
outputs and a few flags. fp16 tensors are stored as float16 and bf16 tensors
as their raw 16-bit patterns (uint16); ``lse`` is float32.
"""

from __future__ import annotations

import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402


@triton.jit
def _tanh(x):
    """tanh from its definition; stands in for Ascend's ``tl.tanh``."""
    e = tl.exp(-2.0 * tl.abs(x))
    t = (1.0 - e) / (1.0 + e)
    return tl.where(x >= 0, t, -t)


def load_reference(path: str):
    sys.modules.setdefault("torch_npu", types.ModuleType("torch_npu"))
    for name in ("triton.language.extra.ascend",
                 "triton.language.extra.ascend.libdevice"):
        sys.modules.setdefault(name, types.ModuleType(name))

    tl.tanh = _tanh
    sys.path.insert(0, path)
    import npu_flash_attention as ref  # the reference module itself
    return ref


DT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}

# (name, dtype, B, Hq, Hkv, Sq, Sk, D, kwargs, with_bwd, flags)
# Names follow the reference's own test IDs where a case mirrors one
# (test/test_comprehensive.py, test/test_bf16_full.py, test/test_real_world.py).
CASES = [
    ("A01_full_fp32", "fp32", 1, 1, 1, 64, 128, 32, {}, True, []),
    ("A03_causal_fp32", "fp32", 1, 1, 1, 128, 128, 32, {"causal": True}, True, []),
    ("A04_causal_fp16", "fp16", 1, 1, 1, 128, 128, 64, {"causal": True}, True, []),
    ("A05_causal_bf16", "bf16", 1, 1, 1, 128, 128, 64, {"causal": True}, True, []),
    ("A09_gqa_hkv2_fp16", "fp16", 1, 4, 2, 64, 64, 64, {"causal": True}, True, []),
    ("B04_gqa4_fp32", "fp32", 1, 4, 1, 64, 64, 32, {"causal": True}, True, []),
    ("A11_window64_fp32", "fp32", 1, 1, 1, 160, 160, 32,
     {"causal": True, "sliding_window": 64}, True, []),
    ("B05_window32_fp32", "fp32", 1, 1, 1, 96, 96, 32,
     {"causal": True, "sliding_window": 32}, True, []),
    ("window_noncausal_fp32", "fp32", 1, 1, 1, 128, 128, 32,
     {"sliding_window": 20}, True, ["ref_kv_tail_bug"]),
    ("A14_sq_lt_sk_fp16", "fp16", 1, 1, 1, 64, 128, 64, {"causal": True}, True, []),
    ("sq_gt_sk_causal_fp32", "fp32", 1, 1, 1, 96, 64, 32, {"causal": True}, True, []),
    ("D02_s33_fp16", "fp16", 1, 1, 1, 33, 33, 64, {"causal": True}, True, []),
    ("D03_s1_fp16", "fp16", 1, 1, 1, 1, 1, 64, {"causal": True}, True, []),
    ("D06_d32_fp16", "fp16", 1, 1, 1, 128, 128, 32, {"causal": True}, True, []),
    ("d128_causal_bf16", "bf16", 1, 2, 1, 64, 64, 128, {"causal": True}, True, []),
    ("F05_scale0.1_fp32", "fp32", 1, 1, 1, 64, 64, 64,
     {"causal": True, "scale": 0.1}, True, []),
    ("softcap20_fp32", "fp32", 1, 2, 1, 96, 96, 32,
     {"causal": True, "soft_cap": 20.0}, True, []),
    ("softcap5_noncausal_fp32", "fp32", 1, 1, 1, 64, 64, 64,
     {"soft_cap": 5.0, "scale": 0.5}, True, []),
    ("alibi_causal_fp32", "fp32", 1, 4, 2, 64, 64, 32,
     {"causal": True, "alibi": True}, True, ["ref_bwd_ignores_alibi"]),
    ("gemma_like_bf16", "bf16", 1, 4, 2, 96, 96, 32,
     {"causal": True, "sliding_window": 48, "soft_cap": 30.0}, True, []),
    ("all_flags_fp16", "fp16", 2, 2, 1, 80, 80, 32,
     {"causal": True, "sliding_window": 40, "soft_cap": 15.0, "alibi": True},
     True, ["ref_bwd_ignores_alibi"]),
    ("kv_tail_noncausal_fp32", "fp32", 1, 1, 1, 64, 96, 64, {}, False,
     ["ref_kv_tail_bug"]),
]


def alibi_slopes(hq: int) -> torch.Tensor:
    """ALiBi slopes 2^(-8(i+1)/Hq), the BASELINE.json config-5 formula."""
    return torch.tensor([2.0 ** (-8.0 * (i + 1) / hq) for i in range(hq)],
                        dtype=torch.float32)


def _store(t: torch.Tensor) -> np.ndarray:
    """Native-width storage: bf16 keeps its bit pattern as uint16."""
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def run_case(ref, case, seed):
    name, dts, b, hq, hkv, sq, sk, d, kw, with_bwd, flags = case
    dt = DT[dts]
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, hq, sq, d, generator=g).to(dt)
    k = torch.randn(b, hkv, sk, d, generator=g).to(dt)
    v = torch.randn(b, hkv, sk, d, generator=g).to(dt)
    go = torch.randn(b, hq, sq, d, generator=g).to(dt)
    kw = dict(kw)
    slopes = None
    if kw.pop("alibi", False):
        slopes = alibi_slopes(hq)
    if dt == torch.bfloat16:
        flags = flags + ["ref_computed_in_fp32"]
        rq, rk, rv, rgo = q.float(), k.float(), v.float(), go.float()
    else:
        rq, rk, rv, rgo = q, k, v, go
    o, lse = ref.npu_flash_attention_forward(
        rq, rk, rv, alibi_slope=slopes, return_lse=True, **kw)
    rec = {"q": _store(q), "k": _store(k), "v": _store(v), "o": _store(o),
           "lse": lse.float().numpy()}
    if slopes is not None:
        rec["alibi_slope"] = slopes.numpy()
    if with_bwd:
        dq, dk, dv = ref.npu_flash_attention_backward(
            rq, rk, rv, o, lse, rgo, alibi_slope=slopes, **kw)
        rec.update(grad_out=_store(go), dq=_store(dq), dk=_store(dk),
                   dv=_store(dv))
    meta = {"name": name, "dtype": dts, "causal": bool(kw.get("causal", False)),
            "sliding_window": int(kw.get("sliding_window", 0)),
            "soft_cap": float(kw.get("soft_cap", 0.0)),
            "scale": kw.get("scale", None), "flags": flags, "seed": seed}
    return rec, meta


def main():
    ref_path = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NPU_FLEX_ATT_REFERENCE")
    if not ref_path:
        sys.exit("usage: make_golden.py REFERENCE_CHECKOUT [out.npz] "
                 "(or set NPU_FLEX_ATT_REFERENCE)")
    out = sys.argv[2] if len(sys.argv) > 2 else os.path.join(
        os.path.dirname(os.path.abspath(__file__)), "reference_cases.npz")
    ref = load_reference(ref_path)
    arrays = {}
    metas = []
    for idx, case in enumerate(CASES):
        rec, meta = run_case(ref, case, seed=1000 + idx)
        for key, val in rec.items():
            arrays[f"{meta['name']}/{key}"] = val
        metas.append(meta)
        print("generated", meta["name"], flush=True)
    import json
    arrays["__meta__"] = np.frombuffer(json.dumps(metas).encode(), dtype=np.uint8)
    np.savez_compressed(out, **arrays)
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
