"""Pin the CPU oracle against the reference's own kernel outputs (CPU only).

The golden vectors come from running npu_flash_attention.py's Triton kernels
under Triton's CPU interpreter (tests/golden/make_golden.py). Agreement here is
what lets the GPU parity tests trust the oracle.
"""
import pytest
import torch

from golden_cases import load_cases
from oracle.attention_math import (attention_backward, attention_forward,
                                   attention_forward_reference_tiles)

CASES = load_cases()
IDS = [m["name"] for m, _ in CASES]

# Oracle (fp64 math) vs reference kernel (fp32 accumulate, P rounded to the
# input dtype before P·V). Absolute tolerances per input dtype.
FWD_TOL = {"fp32": 1e-4, "fp16": 1e-2, "bf16": 2e-2}
LSE_TOL = {"fp32": 1e-4, "fp16": 1e-3, "bf16": 1e-3}
BWD_TOL = {"fp32": 1e-4, "fp16": 2e-2, "bf16": 6e-2}


def _dtype_class(meta):
    """bf16 cases ran the reference at fp32 (see make_golden.py)."""
    return "fp32" if "ref_computed_in_fp32" in meta["flags"] else meta["dtype"]


def _kwargs(meta, rec):
    return dict(causal=meta["causal"], sliding_window=meta["sliding_window"],
                soft_cap=meta["soft_cap"], scale=meta["scale"],
                alibi_slope=rec.get("alibi_slope"))


def _max_abs(a, b):
    a, b = a.double(), b.double()
    finite = torch.isfinite(b)
    assert torch.equal(torch.isfinite(a), finite)
    return (a[finite] - b[finite]).abs().max().item() if finite.any() else 0.0


@pytest.mark.parametrize("meta,rec", CASES, ids=IDS)
def test_forward_matches_reference(meta, rec):
    o, lse = attention_forward(rec["q"], rec["k"], rec["v"], **_kwargs(meta, rec))
    dt = _dtype_class(meta)
    # The tile-walk restatement reproduces the reference in every case,
    # including the ones where its padded keys leak into the softmax.
    o_t, lse_t = attention_forward_reference_tiles(rec["q"], rec["k"], rec["v"],
                                                   **_kwargs(meta, rec))
    assert _max_abs(o_t, rec["o"]) < FWD_TOL[dt]
    assert _max_abs(lse_t, rec["lse"]) < LSE_TOL[dt] * max(1.0, rec["lse"].abs().max().item())
    if "ref_kv_tail_bug" in meta["flags"]:
        # The reference keeps padded key columns (logit 0) in its non-causal
        # path; the math path has no such columns, so the two must differ.
        assert _max_abs(o, rec["o"].double()) > 1e-3
        return
    assert _max_abs(o, rec["o"]) < FWD_TOL[dt]
    assert _max_abs(lse, rec["lse"]) < LSE_TOL[dt] * max(1.0, rec["lse"].abs().max().item())


@pytest.mark.parametrize("meta,rec", [c for c in CASES if "dq" in c[1]],
                         ids=[m["name"] for m, r in CASES if "dq" in r])
def test_backward_matches_reference(meta, rec):
    kw = _kwargs(meta, rec)
    dt = _dtype_class(meta)
    ignores_alibi = "ref_bwd_ignores_alibi" in meta["flags"]
    # Backward from the reference's own forward output and LSE, as its
    # autograd function does (npu_flash_attention.py:762,774).
    dq, dk, dv = attention_backward(
        rec["q"], rec["k"], rec["v"], rec["grad_out"], out=rec["o"],
        lse=rec["lse"], alibi_in_backward=not ignores_alibi, **kw)
    scale_ref = max(1.0, max(rec[n].double().abs().max().item() for n in ("dq", "dk", "dv")))
    tol = BWD_TOL[dt] * scale_ref
    assert _max_abs(dq, rec["dq"]) < tol
    assert _max_abs(dk, rec["dk"]) < tol
    assert _max_abs(dv, rec["dv"]) < tol
    if ignores_alibi:
        # The true gradient of the reference forward differs from what the
        # reference kernels return; the build ships the true gradient.
        dq_true, _, _ = attention_backward(rec["q"], rec["k"], rec["v"],
                                           rec["grad_out"], **kw)
        assert _max_abs(dq_true, rec["dq"]) > 2 * tol


def test_oracle_backward_is_autograd_of_forward():
    """The closed-form oracle backward equals autograd through the oracle forward."""
    g = torch.Generator().manual_seed(7)
    b, hq, hkv, s, d = 1, 4, 2, 40, 16
    q = torch.randn(b, hq, s, d, generator=g, dtype=torch.float64)
    k = torch.randn(b, hkv, s, d, generator=g, dtype=torch.float64)
    v = torch.randn(b, hkv, s, d, generator=g, dtype=torch.float64)
    go = torch.randn(b, hq, s, d, generator=g, dtype=torch.float64)
    slopes = torch.tensor([0.5, 0.25, 0.125, 0.0625], dtype=torch.float64)
    kw = dict(causal=True, sliding_window=9, soft_cap=3.0, alibi_slope=slopes, scale=0.3)
    qr, kr, vr = (x.clone().requires_grad_(True) for x in (q, k, v))
    o, _ = attention_forward(qr, kr, vr, **kw)
    o.backward(go)
    dq, dk, dv = attention_backward(q, k, v, go, **kw)
    for a, b_ in ((dq, qr.grad), (dk, kr.grad), (dv, vr.grad)):
        assert (a - b_).abs().max().item() < 1e-10


FP16_BWD = [c for c in CASES if "dq" in c[1] and _dtype_class(c[0]) == "fp16"
            and "ref_bwd_ignores_alibi" not in c[0]["flags"]]


@pytest.mark.parametrize("meta,rec", FP16_BWD, ids=[m["name"] for m, _ in FP16_BWD])
def test_operand_casts_restate_reference_kernels(meta, rec):
    """With P and dS rounded to fp16 before the gradient products (as the
    reference kernels round them) the oracle lands closer to the reference's
    own fp16 gradients than the all-fp64 oracle does."""
    kw = _kwargs(meta, rec)
    args = (rec["q"], rec["k"], rec["v"], rec["grad_out"])
    plain = attention_backward(*args, out=rec["o"], lse=rec["lse"], **kw)
    cast = attention_backward(*args, out=rec["o"], lse=rec["lse"],
                              operand_dtype=torch.float16, **kw)
    for name, a, c in zip(("dq", "dk", "dv"), plain, cast):
        r = rec[name].double()
        rel_plain = ((a - r).abs() / (1 + r.abs())).max().item()
        rel_cast = ((c - r).abs() / (1 + r.abs())).max().item()
        rms_plain = (a - r).pow(2).mean().sqrt().item()
        rms_cast = (c - r).pow(2).mean().sqrt().item()
        assert rel_cast <= rel_plain + 1e-9, (name, rel_cast, rel_plain)
        assert rms_cast <= rms_plain + 1e-9, (name, rms_cast, rms_plain)
        assert rel_cast < 1e-3, (name, rel_cast)
