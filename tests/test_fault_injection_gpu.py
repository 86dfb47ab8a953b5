"""Failure detection on the GPU without a GPU fault.

The tcgen05 kernels bound every mbarrier wait. With the test-only flag
BFA_DEBUG_INJECT_STALL one softmax wait targets a barrier that nothing ever
completes; the wait runs out after a short limit, the CTA drains its async
copies and MMAs, frees TMEM, and the kernel returns with
BFA_ERR_DEVICE_TIMEOUT in the status word. The context stays usable.
"""
import pytest
import torch

import bfa_lib
import npu_flash_attention as nfa
from oracle.attention_math import attention_forward

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _qkv(seed=0, s=512, d=128):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(1, 2, s, d, generator=g).to(torch.bfloat16) for _ in range(3)]


def test_injected_stall_reports_timeout_and_context_survives():
    q, k, v = _qkv()
    qd, kd, vd = (t.to(DEV) for t in (q, k, v))
    nfa.check_device_status(DEV)  # start clean
    nfa.npu_flash_attention_forward(qd, kd, vd, causal=True, _wait_timeout_ns=20_000_000,
                                    _debug_flags=bfa_lib.DEBUG_INJECT_STALL)
    torch.cuda.synchronize()
    code = bfa_lib.read_and_clear_status(torch.device(DEV))
    assert code == bfa_lib.ERR_DEVICE_TIMEOUT
    # The same context keeps working and gives correct results.
    o = nfa.npu_flash_attention_forward(qd, kd, vd, causal=True)
    o_ref, _ = attention_forward(q, k, v, causal=True)
    assert (o.cpu().double() - o_ref).abs().max().item() < 2e-2
    nfa.check_device_status(DEV)


def test_injected_stall_in_backward_kernels():
    """Both tcgen05 backward kernels stall on their first elementwise wait,
    time out, clean up and report; the next backward is correct."""
    q, k, v = _qkv(2)
    go = _qkv(3)[0]
    qd, kd, vd, god = (t.to(DEV) for t in (q, k, v, go))
    o, lse = nfa.npu_flash_attention_forward(qd, kd, vd, causal=True, return_lse=True)
    nfa.check_device_status(DEV)
    nfa.npu_flash_attention_backward(qd, kd, vd, o, lse, god, causal=True,
                                     _wait_timeout_ns=20_000_000,
                                     _debug_flags=bfa_lib.DEBUG_INJECT_STALL)
    torch.cuda.synchronize()
    assert bfa_lib.read_and_clear_status(torch.device(DEV)) == bfa_lib.ERR_DEVICE_TIMEOUT
    from oracle.attention_math import reference_backward
    dq, dk, dv = nfa.npu_flash_attention_backward(qd, kd, vd, o, lse, god, causal=True)
    rq, rk, rv = reference_backward(q, k, v, go, causal=True)
    for a, r in ((dq, rq), (dk, rk), (dv, rv)):
        assert ((a.cpu().double() - r).abs() / (1 + r.abs())).max().item() < 2e-2
    nfa.check_device_status(DEV)


def test_check_device_status_raises_on_timeout():
    q, k, v = (t.to(DEV) for t in _qkv(1))
    nfa.npu_flash_attention_forward(q, k, v, causal=True, _wait_timeout_ns=20_000_000,
                                    _debug_flags=bfa_lib.DEBUG_INJECT_STALL)
    with pytest.raises(RuntimeError, match="timed out"):
        nfa.check_device_status(DEV)
    nfa.check_device_status(DEV)  # cleared
