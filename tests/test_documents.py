"""Document masking on the CPU: the oracle's keep-mask extension equals
attention computed document by document, and the host API builds the
per-position document bounds the kernels read (no GPU needed)."""
import pytest
import torch

import npu_flash_attention as nfa
from oracle.attention_math import attention_backward, attention_forward


@pytest.mark.parametrize("causal,window", [(True, 0), (False, 0), (True, 5)])
def test_oracle_document_mask_is_blockwise_attention(causal, window):
    g = torch.Generator().manual_seed(1)
    q, k, v, go = (torch.randn(1, 2, 90, 16, generator=g) for _ in range(4))
    cu = [0, 30, 31, 90]
    kw = dict(causal=causal, sliding_window=window)
    o, lse = attention_forward(q, k, v, cu_seqlens=torch.tensor(cu), **kw)
    dq, dk, dv = attention_backward(q, k, v, go, cu_seqlens=torch.tensor(cu), **kw)
    for a, b in zip(cu[:-1], cu[1:]):
        s = slice(a, b)
        o_s, lse_s = attention_forward(q[:, :, s], k[:, :, s], v[:, :, s], **kw)
        dq_s, dk_s, dv_s = attention_backward(q[:, :, s], k[:, :, s], v[:, :, s], go[:, :, s], **kw)
        assert torch.allclose(o[:, :, s], o_s, atol=1e-12)
        assert torch.allclose(lse[:, :, s], lse_s, atol=1e-12)
        for x, y in ((dq, dq_s), (dk, dk_s), (dv, dv_s)):
            assert torch.allclose(x[:, :, s], y, atol=1e-12)


def test_document_bounds_per_position():
    start, end = nfa._documents(torch.tensor([0, 3, 3, 7]), 7, "cpu")
    assert start.tolist() == [0, 0, 0, 3, 3, 3, 3]
    assert end.tolist() == [3, 3, 3, 7, 7, 7, 7]
    assert start.dtype == torch.int32 and end.dtype == torch.int32


@pytest.mark.parametrize("cu,positions", [([1, 5], 4), ([0, 5, 3], 3), ([0], 0), ([0, 4], 5)])
def test_document_bounds_reject_bad_cu_seqlens(cu, positions):
    with pytest.raises(ValueError):
        nfa._documents(torch.tensor(cu), positions, "cpu")
