"""GPU parity of document masking (``cu_seqlens``): packed variable-length
sequences where a pair is kept only inside one document, on top of the
causal / window masks. The reference has no document mask (its README lists
document / block masks as missing); the oracle's keep-mask extension defines
it, and the oracle itself is checked on the CPU (test_documents.py) to equal
attention run document by document.

Every path is covered: the tcgen05 kernels (head_dim 64 / 128 / 256), the
generic fp32 kernels, and the split-KV decoding path.
"""
import pytest
import torch

import npu_flash_attention as nfa
from oracle.attention_math import attention_forward
from test_parity_gpu import DEV, LSE_RTOL, TOL, _err, _inputs, _lse_err, check_case

pytestmark = pytest.mark.gpu

CASES = [
    # (dtype, d, hq, hkv, s, cu_seqlens, mask)
    (torch.bfloat16, 128, 8, 2, 700, [0, 100, 101, 350, 700], dict(causal=True)),
    (torch.bfloat16, 128, 4, 4, 640, [0, 128, 256, 640], dict(causal=True)),
    (torch.float16, 64, 4, 2, 513, [0, 200, 513], dict()),
    (torch.bfloat16, 128, 4, 1, 600, [0, 37, 290, 600], dict(causal=True, sliding_window=64)),
    (torch.bfloat16, 256, 4, 2, 520, [0, 260, 520], dict(causal=True, soft_cap=30.0)),
    (torch.float32, 64, 2, 2, 300, [0, 150, 300], dict(causal=True)),
    (torch.bfloat16, 128, 4, 2, 400, [0, 10, 20, 400], dict(causal=True, alibi=True)),
    (torch.bfloat16, 128, 4, 2, 333, [0, 100, 333], dict(causal=True, alibi=True, sliding_window=64)),
    (torch.bfloat16, 256, 4, 2, 300, [0, 50, 300], dict(causal=True, alibi=True, sliding_window=100)),
    (torch.float16, 64, 2, 1, 257, [0, 3, 257], dict(alibi=True)),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "{}-d{}-h{}-{}-s{}-docs{}-{}".format(
    str(c[0]).split(".")[-1], c[1], c[2], c[3], c[4], len(c[5]) - 1, "-".join(sorted(c[6])) or "full"))
def test_document_mask(case):
    dt, d, hq, hkv, s, cu, mask = case
    mask = dict(mask)
    if mask.pop("alibi", False):
        mask["alibi_slope"] = torch.tensor([2.0 ** (-8.0 * (i + 1) / hq) for i in range(hq)])
    q, k, v, go = _inputs(s + d, 1, hq, hkv, s, s, d, dt)
    check_case(q, k, v, go, cu_seqlens=torch.tensor(cu), **mask)


def test_document_mask_decode_path():
    """Few query rows per KV head (the split-KV decoding path), queries at the
    end of the keys, the last document starting inside the key range."""
    q, k, v, _ = _inputs(9, 2, 8, 2, 2, 3000, 128, torch.bfloat16)
    cu = torch.tensor([0, 1000, 2500, 3000])
    kw = dict(causal=True, cu_seqlens=cu)
    o, lse = nfa.npu_flash_attention_forward(q.to(DEV), k.to(DEV), v.to(DEV), return_lse=True,
                                             q_pos_offset=2998, **kw)
    o_ref, lse_ref = attention_forward(q, k, v, q_offset=2998, **kw)
    assert _err(o, o_ref) < TOL[torch.bfloat16]
    assert _lse_err(lse, lse_ref) < LSE_RTOL


def test_document_mask_through_flex_attention():
    """AttentionConfig.cu_seqlens through the autograd path."""
    q, k, v, go = _inputs(4, 1, 4, 2, 384, 384, 128, torch.bfloat16)
    qd, kd, vd = (t.to(DEV).requires_grad_(True) for t in (q, k, v))
    cu = torch.tensor([0, 200, 384])
    out = nfa.flex_attention(qd, kd, vd, config=nfa.AttentionConfig(causal=True, cu_seqlens=cu))
    out.backward(go.to(DEV))
    # Same as two separate calls, one per document.
    parts = []
    for a, b in ((0, 200), (200, 384)):
        qs, ks, vs = (t[:, :, a:b].to(DEV).requires_grad_(True) for t in (q, k, v))
        o_s = nfa.flex_attention(qs, ks, vs, causal=True)
        o_s.backward(go[:, :, a:b].to(DEV))
        parts.append((o_s, qs.grad, ks.grad, vs.grad))
    for i, full in enumerate((out, qd.grad, kd.grad, vd.grad)):
        ref = torch.cat([p_[i] for p_ in parts], 2)
        assert _err(full, ref.float().cpu().double()) < TOL[torch.bfloat16]
