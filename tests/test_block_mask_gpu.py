"""GPU parity of block-sparse masks (``block_mask``): only the 128x128 blocks
of the score matrix that the mask marks are computed, on top of the causal /
window / document masks. The reference has no block mask (its README lists
document / block masks as missing); the oracle's block keep-mask defines it
and is checked on the CPU against a plain masked softmax (test_block_mask.py).

Every path is covered: the tcgen05 kernels (head_dim 64 / 128 / 256, whose
loops skip the blocks that are off), the generic fp32 kernels and the
split-KV decoding path; rows that keep no key give O = 0, LSE = -inf and
zero gradients.
"""
import pytest
import torch

import npu_flash_attention as nfa
from oracle.attention_math import attention_forward
from test_parity_gpu import DEV, LSE_RTOL, TOL, _err, _inputs, _lse_err, check_case

pytestmark = pytest.mark.gpu


def _mask(seed, shape, p_on=0.6, empty_row=None):
    g = torch.Generator().manual_seed(seed)
    m = torch.rand(*shape, generator=g) < p_on
    if empty_row is not None:
        m[..., empty_row, :] = False
    return m


CASES = [
    # (dtype, d, b, hq, hkv, s, mask shape (None = [b, hq, nq, nk]), empty block row, options)
    (torch.bfloat16, 128, 2, 8, 2, 700, None, 2, dict(causal=True)),
    (torch.float16, 64, 1, 4, 2, 513, "heads", None, dict()),
    (torch.bfloat16, 128, 1, 4, 4, 1024, "shared", 1, dict()),
    (torch.bfloat16, 128, 1, 4, 1, 600, None, None, dict(causal=True, sliding_window=200)),
    (torch.bfloat16, 128, 1, 4, 2, 640, None, 0, dict(causal=True, alibi=True, soft_cap=30.0)),
    (torch.bfloat16, 128, 1, 4, 2, 700, None, None, dict(causal=True, docs=[0, 300, 301, 700])),
    (torch.bfloat16, 256, 1, 4, 2, 520, None, 1, dict(causal=True, soft_cap=30.0)),
    (torch.bfloat16, 256, 2, 4, 2, 640, "heads", None, dict(alibi=True)),
    (torch.float16, 256, 1, 2, 1, 400, None, None, dict(causal=True, docs=[0, 130, 400])),
    (torch.float32, 64, 1, 2, 2, 300, None, 1, dict(causal=True)),
]


def _shape(kind, b, hq, s):
    n = -(-s // 128)
    return {"heads": (hq, n, n), "shared": (n, n)}.get(kind, (b, hq, n, n))


@pytest.mark.parametrize("case", CASES, ids=lambda c: "{}-d{}-b{}-h{}-{}-s{}-{}-{}".format(
    str(c[0]).split(".")[-1], c[1], c[2], c[3], c[4], c[5], c[6] or "full",
    "-".join(sorted(c[8])) or "nomask"))
def test_block_mask(case):
    dt, d, b, hq, hkv, s, kind, empty, opts = case
    opts = dict(opts)
    if opts.pop("alibi", False):
        opts["alibi_slope"] = torch.tensor([2.0 ** (-8.0 * (i + 1) / hq) for i in range(hq)])
    docs = opts.pop("docs", None)
    if docs is not None:
        opts["cu_seqlens"] = torch.tensor(docs)
    m = _mask(s + d + b, _shape(kind, b, hq, s), empty_row=empty)
    q, k, v, go = _inputs(s + d, b, hq, hkv, s, s, d, dt)
    check_case(q, k, v, go, block_mask=m, **opts)


def test_block_mask_decode_path():
    """Few query rows per KV head (the split-KV decoding path): the keys of
    the off blocks are dropped, the rest is plain attention."""
    q, k, v, _ = _inputs(11, 2, 8, 2, 2, 3000, 128, torch.bfloat16)
    m = _mask(5, (1, 8, 1, 24))
    m[0, 3] = False  # a head that sees no key
    o, lse = nfa.npu_flash_attention_forward(q.to(DEV), k.to(DEV), v.to(DEV), return_lse=True,
                                             block_mask=m.to(DEV))
    o_ref, lse_ref = attention_forward(q, k, v, block_mask=m)
    assert _err(o, o_ref) < TOL[torch.bfloat16]
    assert _lse_err(lse, lse_ref) < LSE_RTOL
    assert torch.isneginf(lse[:, 3]).all().item()


def test_block_diagonal_mask_is_separate_calls():
    """A block-diagonal mask over 128-token blocks through flex_attention and
    autograd equals one independent call per block."""
    q, k, v, go = _inputs(7, 1, 4, 2, 384, 384, 128, torch.bfloat16)
    qd, kd, vd = (t.to(DEV).requires_grad_(True) for t in (q, k, v))
    cfg = nfa.AttentionConfig(causal=True, block_mask=torch.eye(3, dtype=torch.bool))
    out = nfa.flex_attention(qd, kd, vd, config=cfg)
    out.backward(go.to(DEV))
    parts = []
    for a in (0, 128, 256):
        qs, ks, vs = (t[:, :, a:a + 128].to(DEV).requires_grad_(True) for t in (q, k, v))
        o_s = nfa.flex_attention(qs, ks, vs, causal=True)
        o_s.backward(go[:, :, a:a + 128].to(DEV))
        parts.append((o_s, qs.grad, ks.grad, vs.grad))
    for i, full in enumerate((out, qd.grad, kd.grad, vd.grad)):
        ref = torch.cat([p_[i] for p_ in parts], 2)
        assert _err(full, ref.float().cpu().double()) < TOL[torch.bfloat16]


@pytest.mark.parametrize("d", [128, 256])
def test_sparse_mask_skips_work(d):
    """A mask that keeps the diagonal block row only must not cost the dense
    time: the kernels' loops visit the blocks that are on. (Timing bound is
    loose: half the dense causal forward. S = 16384, so that the dense work,
    quadratic in S, is well above the per-tile cost both share: loading Q and
    storing O and the LSE.)"""
    B, H, S = 1, 16, 16384
    q = torch.randn(B, H, S, d, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(B, H, S, d, device=DEV, dtype=torch.bfloat16)
    v = torch.randn_like(k)
    n = S // 128
    m = torch.eye(n, dtype=torch.bool, device=DEV)

    def run(mask):
        for _ in range(2):
            nfa.npu_flash_attention_forward(q, k, v, causal=True, block_mask=mask)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            nfa.npu_flash_attention_forward(q, k, v, causal=True, block_mask=mask)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 5

    dense, sparse = run(None), run(m)
    assert sparse < 0.5 * dense, (sparse, dense)
    nfa.check_device_status(DEV)
