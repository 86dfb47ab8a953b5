"""GPU parity: the CUDA kernels vs the CPU oracle on identical seeded inputs.

Tolerances (absolute, from the build's contract): fp32 1e-4, fp16 1e-2,
bf16 2e-2 for outputs and gradients; LSE 1e-3 relative. Case names follow the
reference tests they mirror (test/test_comprehensive.py A/B/C/D/F,
test/test_real_world.py R, test/test_supplementary.py S).
"""
import math

import pytest
import torch

import npu_flash_attention as nfa
from golden_cases import load_cases
from oracle.attention_math import attention_backward, attention_forward, reference_backward

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.float16: 1e-2, torch.bfloat16: 2e-2}
LSE_RTOL = 1e-3
DEV = "cuda:0"


def _inputs(seed, b, hq, hkv, sq, sk, d, dtype, scale_in=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(b, hq, sq, d, generator=g) * scale_in).to(dtype)
    k = (torch.randn(b, hkv, sk, d, generator=g) * scale_in).to(dtype)
    v = torch.randn(b, hkv, sk, d, generator=g).to(dtype)
    go = torch.randn(b, hq, sq, d, generator=g).to(dtype)
    return q, k, v, go


def _err(a, ref):
    """Largest |a − ref| / (1 + |ref|): below `tol` exactly when
    torch.allclose(a, ref, atol=tol, rtol=tol) holds, the form the reference's
    own tests use (e.g. test/test_bf16_full.py with TOL_FWD = 2e-2). A pure
    absolute bound is not attainable for 16-bit outputs above ~5 (half an
    ulp of bf16 at 8 is 0.031)."""
    a = a.detach().cpu().double()
    ref = ref.double()
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(a), fin), "inf/nan pattern differs"
    if not fin.any():
        return 0.0
    return ((a[fin] - ref[fin]).abs() / (1.0 + ref[fin].abs())).max().item()


def _lse_err(lse, ref):
    lse = lse.detach().cpu().double()
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(lse), fin)
    if not fin.any():
        return 0.0
    return ((lse[fin] - ref[fin]).abs() / ref[fin].abs().clamp_min(1.0)).max().item()


def check_case(q, k, v, go, *, tol=None, bwd=True, **kw):
    dtype = q.dtype
    tol = tol or TOL[dtype]
    alibi = kw.get("alibi_slope")
    kw_dev = dict(kw)
    if alibi is not None:
        kw_dev["alibi_slope"] = alibi.to(DEV)
    qd, kd, vd, god = (t.to(DEV) for t in (q, k, v, go))
    o, lse = nfa.npu_flash_attention_forward(qd, kd, vd, return_lse=True, **kw_dev)
    o_ref, lse_ref = attention_forward(q, k, v, **kw)
    assert o.dtype == dtype and lse.dtype == torch.float32
    assert o.shape == q.shape and lse.shape == q.shape[:3]
    e_o = _err(o, o_ref)
    e_l = _lse_err(lse, lse_ref)
    assert e_o < tol, f"O err {e_o}"
    assert e_l < LSE_RTOL, f"LSE err {e_l}"
    if not bwd:
        return
    dq, dk, dv = nfa.npu_flash_attention_backward(qd, kd, vd, o, lse, god, **kw_dev)
    # The backward is checked as the operator it is: a function of
    # (q, k, v, out, lse, dout), given the same out the kernels got and the
    # exact LSE, with P and dS rounded to the input dtype before the gradient
    # products as the reference kernels round them. (The exact LSE rather than
    # the kernel's fp32 one: at logits near 1e4 an fp32 ulp of the LSE is
    # 1e-3, which the fp64 logits here would not share.)
    op_dt = dtype if dtype in (torch.float16, torch.bfloat16) else None
    dq_r, dk_r, dv_r = attention_backward(q, k, v, go, out=o.cpu(), lse=lse_ref,
                                          operand_dtype=op_dt, **kw)
    assert dq.shape == q.shape and dk.shape == k.shape and dv.shape == v.shape
    for name, a, r in (("dq", dq, dq_r), ("dk", dk, dk_r), ("dv", dv, dv_r)):
        e = _err(a, r)
        assert e < tol, f"{name} err {e}"
    nfa.check_device_status(DEV)


# ---------------------------------------------------------------- golden cases
GOLDEN = load_cases()


@pytest.mark.parametrize("meta,rec", GOLDEN, ids=[m["name"] for m, _ in GOLDEN])
def test_golden_inputs(meta, rec):
    """The golden inputs through the CUDA path, against the oracle (which the
    CPU suite pins to the reference's own kernel outputs)."""
    kw = dict(causal=meta["causal"], sliding_window=meta["sliding_window"],
              soft_cap=meta["soft_cap"], scale=meta["scale"],
              alibi_slope=rec.get("alibi_slope"))
    go = rec.get("grad_out", torch.zeros_like(rec["q"]))
    check_case(rec["q"], rec["k"], rec["v"], go, bwd="dq" in rec, **kw)
    if not meta["flags"]:
        # No divergence expected from the reference itself here either.
        o = nfa.npu_flash_attention_forward(rec["q"].to(DEV), rec["k"].to(DEV), rec["v"].to(DEV),
                                            **{**kw, "alibi_slope": None if kw["alibi_slope"] is None
                                               else kw["alibi_slope"].to(DEV)})
        assert _err(o, rec["o"]) < 2 * TOL[rec["q"].dtype]


# ---------------------------------------------------------------- sweep
SWEEP = []
for dt in (torch.bfloat16, torch.float16, torch.float32):
    for d in (64, 128):
        for causal, window in ((False, 0), (True, 0), (True, 96), (False, 80)):
            SWEEP.append((dt, d, causal, window))


@pytest.mark.parametrize("dt,d,causal,window", SWEEP,
                         ids=[f"{str(a).split('.')[-1]}-d{b}-c{int(c)}-w{w}" for a, b, c, w in SWEEP])
def test_mask_dtype_headdim_sweep(dt, d, causal, window):
    q, k, v, go = _inputs(11, 1, 4, 2, 300, 300, d, dt)
    check_case(q, k, v, go, causal=causal, sliding_window=window)


@pytest.mark.parametrize("sq,sk", [(1, 1), (16, 16), (33, 33), (127, 127), (128, 128), (129, 129),
                                   (255, 257), (257, 129), (64, 520), (520, 64), (384, 1000)])
@pytest.mark.parametrize("causal", [False, True])
def test_ragged_lengths_bf16(sq, sk, causal):
    """Lengths that are not tile multiples, incl. Sq != Sk (top-left causal)."""
    q, k, v, go = _inputs(sq * 7 + sk, 2, 2, 1, sq, sk, 128, torch.bfloat16)
    check_case(q, k, v, go, causal=causal)


@pytest.mark.parametrize("d", [16, 32, 64, 96, 128, 256])
def test_head_dims_fp16(d):
    q, k, v, go = _inputs(d, 1, 2, 2, 160, 160, d, torch.float16)
    check_case(q, k, v, go, causal=True)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("d", [64, 128])
def test_softcap_and_alibi(dt, d):
    q, k, v, go = _inputs(5, 1, 4, 1, 333, 333, d, dt)
    slopes = torch.tensor([2.0 ** (-8.0 * (i + 1) / 4) for i in range(4)])
    check_case(q, k, v, go, causal=True, soft_cap=20.0)
    check_case(q, k, v, go, causal=True, alibi_slope=slopes)
    check_case(q, k, v, go, causal=True, sliding_window=50, soft_cap=30.0, alibi_slope=slopes)
    check_case(q, k, v, go, causal=False, soft_cap=5.0, scale=0.3)


@pytest.mark.parametrize("g", [1, 2, 4, 8])
def test_gqa_ratios(g):
    """A06-A09 / B04: GQA ratios 1..8; dK/dV are sums over the group."""
    q, k, v, go = _inputs(g, 2, 2 * g, 2, 256, 256, 128, torch.bfloat16)
    check_case(q, k, v, go, causal=True)


def test_stability_cases():
    """C01-C05: extreme scales and inputs stay finite and correct."""
    q, k, v, go = _inputs(3, 1, 1, 1, 128, 128, 64, torch.float32, scale_in=10.0)
    o = nfa.npu_flash_attention_forward(q.to(DEV), k.to(DEV), v.to(DEV), causal=True, scale=10.0)
    assert torch.isfinite(o).all()
    # Logits reach |u| ~ 1e4 here; one fp32 ulp there is ~1e-3, so fp32
    # arithmetic (the reference's as well) agrees with fp64 only to ~1e-3.
    check_case(q, k, v, go, causal=True, scale=10.0, tol=5e-3)
    check_case(q, k, v, go, causal=True, scale=0.01)
    q16, k16, v16, go16 = _inputs(4, 1, 1, 1, 128, 128, 64, torch.float16, scale_in=100.0)
    o = nfa.npu_flash_attention_forward(q16.to(DEV), k16.to(DEV), v16.to(DEV), causal=True)
    assert torch.isfinite(o).all()
    z = torch.zeros(1, 1, 128, 64)
    o = nfa.npu_flash_attention_forward(q.to(DEV), k.to(DEV), z.to(DEV), causal=True)
    assert o.abs().max().item() < 1e-5
    check_case(z, k, v, go, causal=True)


def test_fully_masked_rows_give_zero_and_neg_inf_lse():
    """Non-causal window with Sq > Sk + W: rows i > Sk-1+W see no key."""
    q, k, v, go = _inputs(9, 1, 2, 2, 200, 64, 128, torch.bfloat16)
    check_case(q, k, v, go, sliding_window=40)
    o, lse = nfa.npu_flash_attention_forward(q.to(DEV), k.to(DEV), v.to(DEV), sliding_window=40,
                                             return_lse=True)
    assert torch.isneginf(lse[:, :, 104:]).all()
    assert (o[:, :, 104:] == 0).all()


def test_noncontiguous_and_strided_inputs():
    """R01-R03, R10, S09: transposed Q, sliced K, stride-0 broadcast K/V, as_strided."""
    g = torch.Generator().manual_seed(1)
    qt = torch.randn(1, 256, 2, 64, generator=g).to(torch.float16).transpose(1, 2)
    kf = torch.randn(1, 2, 512, 64, generator=g).to(torch.float16)
    k = kf[:, :, :256, :]
    v = torch.randn(1, 2, 256, 64, generator=g).to(torch.float16)
    go = torch.randn(1, 2, 256, 64, generator=g).to(torch.float16)
    qd, kd, vd = qt.to(DEV).transpose(1, 2).contiguous().transpose(1, 2), k.to(DEV), v.to(DEV)
    assert not qd.is_contiguous()
    o = nfa.npu_flash_attention_forward(qd, kd, vd, causal=True)
    assert o.stride() == qd.stride()  # empty_like keeps q's layout (:631)
    o_ref, _ = attention_forward(qt, k, v, causal=True)
    assert _err(o, o_ref) < 1e-2
    check_case(qt.contiguous(), k.contiguous(), v, go, causal=True)
    # stride-0 broadcast over heads
    kb = torch.randn(1, 1, 128, 64, generator=g).to(torch.float16)
    vb = torch.randn(1, 1, 128, 64, generator=g).to(torch.float16)
    q4 = torch.randn(1, 4, 128, 64, generator=g).to(torch.float16)
    o = nfa.npu_flash_attention_forward(q4.to(DEV), kb.to(DEV).expand(1, 4, 128, 64),
                                        vb.to(DEV).expand(1, 4, 128, 64), causal=True)
    o_ref, _ = attention_forward(q4, kb, vb, causal=True)
    assert _err(o, o_ref) < 1e-2
    # as_strided view with standard strides
    qa = q4[:, :1].contiguous()
    qs = qa.to(DEV).as_strided(qa.shape, (128 * 64, 64, 64, 1))
    o = nfa.npu_flash_attention_forward(qs, kb.to(DEV), vb.to(DEV), causal=True)
    o_ref, _ = attention_forward(qa, kb, vb, causal=True)
    assert _err(o, o_ref) < 1e-2


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_bitwise_determinism(dt):
    """R06 / R11: identical inputs give bitwise-identical O, LSE, dQ, dK, dV."""
    q, k, v, go = (t.to(DEV) for t in _inputs(42, 1, 8, 2, 640, 640, 128, dt))
    o1, l1 = nfa.npu_flash_attention_forward(q, k, v, causal=True, return_lse=True)
    o2, l2 = nfa.npu_flash_attention_forward(q, k, v, causal=True, return_lse=True)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    g1 = nfa.npu_flash_attention_backward(q, k, v, o1, l1, go, causal=True)
    g2 = nfa.npu_flash_attention_backward(q, k, v, o1, l1, go, causal=True)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def test_autograd_through_flex_attention():
    """F02 / S07: the autograd path gives the oracle's gradients."""
    q, k, v, go = _inputs(8, 2, 8, 2, 200, 200, 128, torch.bfloat16)
    qd, kd, vd = (t.to(DEV).requires_grad_(True) for t in (q, k, v))
    cfg = nfa.AttentionConfig(causal=True, sliding_window=64, soft_cap=30.0)
    out = nfa.flex_attention(qd, kd, vd, config=cfg)
    out.backward(go.to(DEV))
    o_r, _ = attention_forward(q, k, v, causal=True, sliding_window=64, soft_cap=30.0)
    dq, dk, dv = reference_backward(q, k, v, go, causal=True, sliding_window=64, soft_cap=30.0)
    assert _err(out, o_r) < 2e-2
    assert _err(qd.grad, dq) < 2e-2 and _err(kd.grad, dk) < 2e-2 and _err(vd.grad, dv) < 2e-2


def test_calls_from_a_fresh_thread():
    """A thread whose first CUDA work is this library's (as PyTorch's autograd
    device threads can be, when every tensor they touch comes from the caching
    allocator) still gets the device context the tensor-map encoder needs, and
    the same results bit for bit."""
    import threading
    q, k, v, go = (t.to(DEV) for t in _inputs(9, 1, 4, 2, 256, 256, 128, torch.bfloat16))
    o, l = nfa.npu_flash_attention_forward(q, k, v, causal=True, return_lse=True)
    g = nfa.npu_flash_attention_backward(q, k, v, o, l, go, causal=True)
    torch.cuda.synchronize()
    out = {}

    def work():
        try:
            o2, l2 = nfa.npu_flash_attention_forward(q, k, v, causal=True, return_lse=True)
            out["g"] = nfa.npu_flash_attention_backward(q, k, v, o2, l2, go, causal=True)
            out["o"] = o2
            torch.cuda.synchronize()
        except Exception as e:  # reported below, on the test's thread
            out["err"] = e

    th = threading.Thread(target=work)
    th.start()
    th.join()
    assert "err" not in out, out.get("err")
    assert torch.equal(out["o"], o)
    for a, b in zip(out["g"], g):
        assert torch.equal(a, b)


def test_cross_dtype_agreement():
    """S01-S03: fp32, fp16 and bf16 runs of the same data agree within 0.1."""
    q, k, v, _ = _inputs(0, 1, 2, 2, 128, 128, 64, torch.float32)
    outs = [nfa.npu_flash_attention_forward(q.to(DEV, dt), k.to(DEV, dt), v.to(DEV, dt), causal=True).float()
            for dt in (torch.float32, torch.float16, torch.bfloat16)]
    assert (outs[0] - outs[1]).abs().max() < 0.1
    assert (outs[0] - outs[2]).abs().max() < 0.1


def test_no_memory_leak():
    """S06: repeated calls do not grow allocated memory."""
    q, k, v, _ = (t.to(DEV) for t in _inputs(2, 1, 2, 2, 256, 256, 64, torch.float16))
    nfa.npu_flash_attention_forward(q, k, v, causal=True)
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated(DEV)
    for _ in range(10):
        nfa.npu_flash_attention_forward(q, k, v, causal=True)
    torch.cuda.synchronize()
    assert abs(torch.cuda.memory_allocated(DEV) - before) < (1 << 20)


def test_training_loop_decreases_loss():
    """S07: five SGD steps on K/V through the kernels."""
    torch.manual_seed(42)
    q = torch.randn(1, 2, 128, 64, device=DEV)
    k = torch.randn(1, 2, 128, 64, device=DEV)
    v = torch.randn(1, 2, 128, 64, device=DEV)
    target = torch.randn(1, 2, 128, 64, device=DEV)
    losses = []
    for _ in range(5):
        out, lse = nfa.npu_flash_attention_forward(q, k, v, causal=True, return_lse=True)
        losses.append((out - target).pow(2).mean().item())
        g = 2 * (out - target) / out.numel()
        _, dk, dv = nfa.npu_flash_attention_backward(q, k, v, out, lse, g, causal=True)
        k, v = k - 10.0 * dk, v - 10.0 * dv
    assert losses[-1] < losses[0]


D256_CASES = [
    # (dtype, sq, sk, causal, window, cap, alibi)
    (torch.bfloat16, 300, 300, True, 0, 0.0, False),
    (torch.bfloat16, 257, 257, False, 0, 0.0, False),
    (torch.float16, 384, 384, True, 100, 0.0, False),
    (torch.bfloat16, 520, 520, True, 0, 50.0, False),
    (torch.bfloat16, 333, 333, True, 64, 50.0, True),
    (torch.float16, 200, 450, False, 0, 5.0, False),   # cap with |s/cap| > 1/2 (exact tanh path)
    (torch.bfloat16, 129, 1000, True, 0, 0.0, True),
    (torch.bfloat16, 1, 130, False, 0, 0.0, False),
]


@pytest.mark.parametrize("case", D256_CASES, ids=lambda c: "{}-q{}-k{}-c{}-w{}-cap{}-a{}".format(
    str(c[0]).split(".")[-1], *c[1:]))
def test_head_dim_256(case):
    """head_dim 256 (the tcgen05 D=256 forward): masks, soft-cap on both tanh
    paths, ALiBi, GQA 2, ragged and Sq != Sk lengths."""
    dt, sq, sk, causal, window, cap, alibi = case
    q, k, v, go = _inputs(sq + 3 * sk, 1, 4, 2, sq, sk, 256, dt)
    slopes = torch.tensor([2.0 ** (-8.0 * (i + 1) / 4) for i in range(4)]) if alibi else None
    check_case(q, k, v, go, causal=causal, sliding_window=window, soft_cap=cap, alibi_slope=slopes)

