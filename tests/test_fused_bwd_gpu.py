"""The one-kernel backward (opt-in with BFA_BWD_FUSED=1) on the GPU.

dK, dV and dQ come out of one tcgen05 kernel; dQ is added into an fp32 buffer
in a fixed order per query tile. Checked here: the same oracle parity as the
two-kernel backward, bitwise determinism across runs, the accumulate mode
(gradients added into fp32 buffers), and the bounded-wait failure path.
"""
import os

import pytest
import torch

import bfa_lib
import npu_flash_attention as nfa
from oracle.attention_math import attention_backward, attention_forward

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(autouse=True)
def fused_on():
    old = os.environ.get("BFA_BWD_FUSED")
    os.environ["BFA_BWD_FUSED"] = "1"
    yield
    if old is None:
        del os.environ["BFA_BWD_FUSED"]
    else:
        os.environ["BFA_BWD_FUSED"] = old


def _err(a, r):
    a, r = a.detach().cpu().double(), r.double()
    return ((a - r).abs() / (1.0 + r.abs())).max().item()


def _inputs(seed, b, hq, hkv, sq, sk, dtype=torch.bfloat16, d=128):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, hq, sq, d, generator=g).to(dtype)
    k = torch.randn(b, hkv, sk, d, generator=g).to(dtype)
    v = torch.randn(b, hkv, sk, d, generator=g).to(dtype)
    go = torch.randn(b, hq, sq, d, generator=g).to(dtype)
    return q, k, v, go


CASES = [
    ("causal_gqa4", dict(b=2, hq=8, hkv=2, sq=640, sk=640), dict(causal=True)),
    ("full", dict(b=1, hq=4, hkv=4, sq=384, sk=384), dict()),
    ("window", dict(b=1, hq=4, hkv=1, sq=700, sk=700), dict(causal=True, sliding_window=150)),
    ("noncausal_window", dict(b=1, hq=2, hkv=1, sq=300, sk=520), dict(sliding_window=90)),
    ("ragged", dict(b=1, hq=2, hkv=2, sq=257, sk=129), dict(causal=True)),
    ("alibi_cap", dict(b=1, hq=4, hkv=2, sq=512, sk=512),
     dict(causal=True, soft_cap=30.0, alibi_slope=torch.tensor([0.5, 0.25, 0.125, 0.0625]))),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("name,shape,mask", CASES, ids=[c[0] for c in CASES])
def test_fused_backward_matches_oracle(name, shape, mask, dtype):
    q, k, v, go = _inputs(sum(map(ord, name)), dtype=dtype, **shape)
    mdev = {**mask, **({"alibi_slope": mask["alibi_slope"].to(DEV)} if "alibi_slope" in mask else {})}
    qd, kd, vd, god = (t.to(DEV) for t in (q, k, v, go))
    o, lse = nfa.npu_flash_attention_forward(qd, kd, vd, return_lse=True, **mdev)
    launches = bfa_lib.load().bfa_launch_count()
    dq, dk, dv = nfa.npu_flash_attention_backward(qd, kd, vd, o, lse, god, **mdev)
    torch.cuda.synchronize()
    nfa.check_device_status(DEV)
    # Δ, the one-kernel backward and the dQ conversion: three launches.
    assert bfa_lib.load().bfa_launch_count() - launches == 3
    _, lse_ref = attention_forward(q, k, v, **mask)
    rq, rk, rv = attention_backward(q, k, v, go, out=o.cpu(), lse=lse_ref, operand_dtype=dtype,
                                    **mask)
    for n, a, r in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
        assert _err(a, r) < 2e-2, (n, _err(a, r))


def test_fused_backward_is_bitwise_deterministic():
    q, k, v, go = (t.to(DEV) for t in _inputs(5, 2, 8, 2, 1024, 1024))
    o, lse = nfa.npu_flash_attention_forward(q, k, v, causal=True, return_lse=True)
    g1 = nfa.npu_flash_attention_backward(q, k, v, o, lse, go, causal=True)
    g2 = nfa.npu_flash_attention_backward(q, k, v, o, lse, go, causal=True)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)
    # Same gradients as the two-kernel path within bf16 rounding.
    os.environ["BFA_BWD_FUSED"] = "0"
    g3 = nfa.npu_flash_attention_backward(q, k, v, o, lse, go, causal=True)
    for a, b in zip(g1, g3):
        assert _err(a, b.cpu().double()) < 2e-2


def test_fused_accumulate_mode_adds_into_fp32():
    q, k, v, go = (t.to(DEV) for t in _inputs(9, 1, 4, 2, 512, 512))
    o, lse = nfa.npu_flash_attention_forward(q, k, v, causal=True, return_lse=True)
    ref = nfa.npu_flash_attention_backward(q, k, v, o, lse, go, causal=True)
    acc = [torch.full(t.shape, 0.25, device=DEV, dtype=torch.float32) for t in ref]
    nfa.npu_flash_attention_backward(q, k, v, o, lse, go, causal=True,
                                     _outputs=tuple(acc), _accumulate=True)
    torch.cuda.synchronize()
    nfa.check_device_status(DEV)
    for a, r in zip(acc, ref):
        assert _err(a - 0.25, r.cpu().double()) < 1e-2


def test_fused_injected_stall_reports_timeout():
    q, k, v, go = (t.to(DEV) for t in _inputs(3, 1, 2, 2, 512, 512))
    o, lse = nfa.npu_flash_attention_forward(q, k, v, causal=True, return_lse=True)
    nfa.check_device_status(DEV)
    nfa.npu_flash_attention_backward(q, k, v, o, lse, go, causal=True,
                                     _wait_timeout_ns=20_000_000,
                                     _debug_flags=bfa_lib.DEBUG_INJECT_STALL)
    torch.cuda.synchronize()
    assert bfa_lib.read_and_clear_status(torch.device(DEV)) == bfa_lib.ERR_DEVICE_TIMEOUT
    dq, dk, dv = nfa.npu_flash_attention_backward(q, k, v, o, lse, go, causal=True)
    _, lse_ref = attention_forward(q.cpu(), k.cpu(), v.cpu(), causal=True)
    rq, rk, rv = attention_backward(q.cpu(), k.cpu(), v.cpu(), go.cpu(), out=o.cpu(), lse=lse_ref,
                                    operand_dtype=torch.bfloat16, causal=True)
    for a, r in ((dq, rq), (dk, rk), (dv, rv)):
        assert _err(a, r) < 2e-2
    nfa.check_device_status(DEV)
