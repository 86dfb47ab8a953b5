"""bfa_bwd_noalloc: the backward entry point that allocates nothing.

Some callers cannot give the library a workspace: a plugin inside a host
framework that owns all device memory and hands over only the input and
output buffers, or a hot path that must not call cudaMalloc because it can
synchronise the device. bfa_bwd_noalloc keeps the backward's row statistics
in a static device array (2^21 query rows, each head's rows rounded up to 64)
instead. These tests call it through
the C ABI and check it against the regular bfa_bwd entry point.

The file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

import bfa_lib
import npu_flash_attention as nfa

DEV = "cuda:0"
TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def _close(a, ref, tol):
    return ((a.double() - ref.double()).abs() / (1.0 + ref.double().abs())).max().item() < tol


def _problem_and_args(q, k, v, o, lse, do, dq, dk, dv, causal):
    pr = nfa._problem(q, k, causal, 0, None, q.shape[-1] ** -0.5, 0.0)
    args = bfa_lib.BwdArgs()
    args.q, args.k, args.v = bfa_lib.tensor(q), bfa_lib.tensor(k), bfa_lib.tensor(v)
    args.o, args.dout = bfa_lib.tensor(o), bfa_lib.tensor(do)
    args.lse = lse.data_ptr()
    args.dq, args.dk, args.dv = bfa_lib.tensor(dq), bfa_lib.tensor(dk), bfa_lib.tensor(dv)
    return pr, args


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,S", [(torch.bfloat16, 640), (torch.float32, 640), (torch.bfloat16, 600)])
def test_noalloc_backward_matches_bfa_bwd_twice(dtype, S):
    """S=600 is not a multiple of 64, so each head's rows are padded inside
    the static array (row pitch 640) and the second statistic starts past the
    first one's padded rows."""
    lib = bfa_lib.load()
    g = torch.Generator().manual_seed(77)
    B, Hq, Hkv, D = 2, 8, 2, 128
    q = torch.randn(B, Hq, S, D, generator=g).to(dtype).to(DEV)
    k = torch.randn(B, Hkv, S, D, generator=g).to(dtype).to(DEV)
    v = torch.randn(B, Hkv, S, D, generator=g).to(dtype).to(DEV)
    do = torch.randn(B, Hq, S, D, generator=g).to(dtype).to(DEV)
    o, lse = nfa.npu_flash_attention_forward(q, k, v, causal=True, return_lse=True)
    # Reference result from the regular entry point (caller-provided workspace).
    rq, rk, rv = nfa.npu_flash_attention_backward(q, k, v, o, lse, do, causal=True)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    for _ in range(2):  # two calls in a row share (and overwrite) the static scratch
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        pr, args = _problem_and_args(q, k, v, o, lse, do, dq, dk, dv, causal=True)
        rc = lib.bfa_bwd_noalloc(ctypes.byref(pr), ctypes.byref(args), stream)
        assert rc == 0, lib.bfa_strerror(rc).decode()
        torch.cuda.synchronize()
        for a, r in ((dq, rq), (dk, rk), (dv, rv)):
            assert _close(a.cpu(), r.cpu(), TOL[dtype])


def test_noalloc_rejects_problems_beyond_its_scratch():
    """Rejected on the host before any device work (runs without a GPU)."""
    lib = bfa_lib.load()
    pr = bfa_lib.Problem()
    pr.batch, pr.heads_q, pr.heads_kv, pr.seqlen_q, pr.seqlen_k, pr.head_dim = 1, 64, 8, 65536, 65536, 128
    pr.dtype, pr.scale = bfa_lib.DTYPE_BF16, 0.088
    assert pr.batch * pr.heads_q * pr.seqlen_q > bfa_lib.NOALLOC_MAX_ROWS
    rc = lib.bfa_bwd_noalloc(ctypes.byref(pr), ctypes.byref(bfa_lib.BwdArgs()), None)
    assert rc == bfa_lib.ERR_SCRATCH_LIMIT
    assert "2097152" in lib.bfa_strerror(rc).decode()
    assert lib.bfa_bwd_noalloc(None, None, None) == -1


def test_noalloc_limit_edge_and_phase_rule():
    """Host-side checks (no GPU): exactly 2^21 padded rows pass the size
    check (the call then stops at the empty argument block), one more 64-row
    tile does not; a phases mask without the Δ phase is rejected."""
    lib = bfa_lib.load()
    pr = bfa_lib.Problem()
    pr.batch, pr.heads_q, pr.heads_kv, pr.seqlen_k, pr.head_dim = 1, 32, 8, 4096, 128
    pr.dtype, pr.scale = bfa_lib.DTYPE_BF16, 0.088
    pr.seqlen_q = bfa_lib.NOALLOC_MAX_ROWS // 32 - 63  # rounds up to exactly 2^16 rows per head
    assert pr.heads_q * ((pr.seqlen_q + 63) // 64 * 64) == bfa_lib.NOALLOC_MAX_ROWS
    rc = lib.bfa_bwd_noalloc(ctypes.byref(pr), None, None)
    assert rc == -1  # past the size check: rejected for the missing arguments
    pr.seqlen_q += 64
    rc = lib.bfa_bwd_noalloc(ctypes.byref(pr), None, None)
    assert rc == bfa_lib.ERR_SCRATCH_LIMIT
    pr.seqlen_q = 256
    args = bfa_lib.BwdArgs()
    for phases in (bfa_lib.PHASE_DKDV, bfa_lib.PHASE_DQ, bfa_lib.PHASE_DKDV | bfa_lib.PHASE_DQ):
        args.phases = phases
        assert lib.bfa_bwd_noalloc(ctypes.byref(pr), ctypes.byref(args), None) == -1
