"""The forward's epilogue merge (``bfa_fwd_args.accumulate``): a call merges
its own result into a running fp32 (O, LSE) in place.

The keys are cut into chunks with absolute position offsets, as a
context-parallel ring visits them. Merging every chunk's call must give
attention over all keys, checked against the oracle, on every forward path:
the tcgen05 kernels (head dims 64, 128, 256), the generic fp32 kernels, and a
running output whose layout the tcgen05 epilogue does not take (it then runs
on the generic kernels). A row that sees no key of a chunk leaves the running
result as it was; a row that sees none at all ends with O = 0 and LSE = -inf.
The merge of separate calls by ``bfa_merge_partial`` gives the same result
within the 16-bit rounding of its partial outputs.
"""
import pytest
import torch

import context_parallel as cp
import npu_flash_attention as nfa
from oracle.attention_math import attention_forward
from test_parity_gpu import DEV, LSE_RTOL, TOL, _err, _inputs, _lse_err

pytestmark = pytest.mark.gpu

CASES = [
    # (dtype, d, hq, hkv, sq, key chunk bounds, q position offset, position of key 0, options)
    (torch.bfloat16, 128, 4, 2, 300, [0, 256, 300, 700], 400, 0, dict(causal=True)),
    (torch.float16, 64, 4, 1, 257, [0, 128, 512], 0, 0, dict()),
    (torch.bfloat16, 128, 2, 2, 384, [0, 384, 768], 384, 0, dict(causal=True, soft_cap=30.0, alibi=True)),
    (torch.bfloat16, 256, 4, 2, 200, [0, 320, 640], 440, 0, dict(causal=True, sliding_window=300)),
    (torch.float16, 256, 2, 1, 130, [0, 64, 200], 0, 0, dict(causal=True)),
    # Keys start at position 100: query rows 0..99 see no key at all.
    (torch.bfloat16, 64, 2, 2, 260, [0, 128, 256], 0, 100, dict(causal=True)),
    (torch.float32, 64, 2, 1, 100, [0, 150, 300], 200, 0, dict(causal=True)),
]


def _opts(opts, hq, dev):
    opts = dict(opts)
    if opts.pop("alibi", False):
        opts["alibi_slope"] = torch.tensor([2.0 ** (-8.0 * (i + 1) / hq) for i in range(hq)])
    dev_opts = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in opts.items()}
    return opts, dev_opts


def _run_chunks(qd, kd, vd, bounds, q_off, k_base, dev_opts, o_acc, lse_acc):
    for a, b in zip(bounds[:-1], bounds[1:]):
        o, lse = nfa.npu_flash_attention_forward(
            qd, kd[:, :, a:b], vd[:, :, a:b], return_lse=True, q_pos_offset=q_off,
            k_pos_offset=k_base + a, _merge_into=(o_acc, lse_acc), **dev_opts)
        assert o is o_acc and lse is lse_acc


@pytest.mark.parametrize("case", CASES, ids=lambda c: "{}-d{}-h{}-{}-sq{}-sk{}-{}".format(
    str(c[0]).split(".")[-1], c[1], c[2], c[3], c[4], c[5][-1], "-".join(sorted(c[8])) or "full"))
def test_chunked_merge_matches_oracle(case):
    dt, d, hq, hkv, sq, bounds, q_off, k_base, opts = case
    opts, dev_opts = _opts(opts, hq, DEV)
    q, k, v, _ = _inputs(sq + d + hq, 2, hq, hkv, sq, bounds[-1], d, dt)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    o_acc = torch.zeros(2, hq, sq, d, device=DEV, dtype=torch.float32)
    lse_acc = torch.full((2, hq, sq), float("-inf"), device=DEV, dtype=torch.float32)
    _run_chunks(qd, kd, vd, bounds, q_off, k_base, dev_opts, o_acc, lse_acc)
    o_ref, lse_ref = attention_forward(q, k, v, q_offset=q_off, k_offset=k_base, **opts)
    torch.cuda.synchronize()
    nfa.check_device_status(DEV)
    assert _err(o_acc, o_ref) < TOL[dt]
    assert _lse_err(lse_acc, lse_ref) < LSE_RTOL
    dead = torch.isneginf(lse_ref)
    assert (o_acc.cpu()[dead] == 0).all()

    # The same chunks through separate calls and bfa_merge_partial.
    o_sep = torch.zeros_like(o_acc)
    lse_sep = torch.full_like(lse_acc, float("-inf"))
    ops = cp.CudaBlockOps()
    for a, b in zip(bounds[:-1], bounds[1:]):
        o_p, lse_p = nfa.npu_flash_attention_forward(
            qd, kd[:, :, a:b], vd[:, :, a:b], return_lse=True, q_pos_offset=q_off,
            k_pos_offset=k_base + a, **dev_opts)
        ops.merge(o_sep, lse_sep, o_p, lse_p)
    torch.cuda.synchronize()
    assert _err(o_acc, o_sep.cpu().double()) < TOL[dt]
    assert torch.equal(torch.isneginf(lse_acc), torch.isneginf(lse_sep))


def test_merge_into_a_strided_running_output():
    """A running output whose row pitch is not a multiple of 16 bytes (the
    tcgen05 epilogue reads and writes it 16 bytes at a time, so the generic
    kernels merge it): same result as a contiguous one."""
    hq, hkv, sq, d = 4, 2, 200, 128
    q, k, v, _ = _inputs(3, 1, hq, hkv, sq, 512, d, torch.bfloat16)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    big = torch.zeros(1, hq, sq, d + 1, device=DEV, dtype=torch.float32)
    o_s = big[..., :d]
    lse_s = torch.full((1, hq, sq), float("-inf"), device=DEV, dtype=torch.float32)
    o_c = torch.zeros(1, hq, sq, d, device=DEV, dtype=torch.float32)
    lse_c = lse_s.clone()
    for o_acc, lse_acc in ((o_s, lse_s), (o_c, lse_c)):
        _run_chunks(qd, kd, vd, [0, 200, 512], 312, 0, dict(causal=True), o_acc, lse_acc)
    torch.cuda.synchronize()
    assert (big[..., d] == 0).all()  # the column past the view is untouched
    assert torch.allclose(o_s, o_c, atol=2e-3, rtol=2e-3)
    assert torch.allclose(lse_s, lse_c, atol=1e-4, rtol=1e-5)
    o_ref, _ = attention_forward(q, k, v, q_offset=312, causal=True)
    assert _err(o_s, o_ref) < TOL[torch.bfloat16]


def test_merge_into_rejects_wrong_accumulators():
    q = torch.randn(1, 2, 64, 64, device=DEV, dtype=torch.bfloat16)
    lse = torch.full((1, 2, 64), float("-inf"), device=DEV)
    with pytest.raises(ValueError):
        nfa.npu_flash_attention_forward(q, q, q, _merge_into=(torch.zeros_like(q), lse))
    with pytest.raises(ValueError):
        nfa.npu_flash_attention_forward(q, q, q, _merge_into=(q.float(), lse[..., :32]))
