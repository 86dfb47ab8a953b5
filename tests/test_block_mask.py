"""Block-sparse masks on the CPU: the oracle's block keep-mask (128x128 blocks
of the score matrix, broadcast over batch and heads) against a plain
masked softmax written out here, and the autograd plumbing of the extra
argument (no GPU needed)."""
import math

import pytest
import torch

from oracle.attention_math import attention_backward, attention_forward, block_keep


def _dense(q, k, v, keep):
    s = q @ k.transpose(-2, -1) / math.sqrt(q.shape[-1])
    s = s.masked_fill(~keep, float("-inf"))
    lse = torch.logsumexp(s, -1)
    p = torch.where(keep, torch.exp(s - torch.where(torch.isfinite(lse), lse, 0).unsqueeze(-1)), 0)
    return p @ v, lse


def test_block_keep_expands_blocks():
    m = torch.tensor([[1, 0, 1], [0, 1, 0]], dtype=torch.bool)
    keep = block_keep(m, 2, 3, 200, 300)
    assert keep.shape == (2, 3, 200, 300)
    assert keep[1, 2, 0, 0] and not keep[1, 2, 0, 128] and keep[0, 0, 127, 299]
    assert keep[0, 0, 128, 128] and not keep[0, 0, 199, 0] and not keep[0, 0, 199, 299]


@pytest.mark.parametrize("causal", [False, True])
def test_oracle_block_mask_matches_dense(causal):
    g = torch.Generator().manual_seed(3)
    b, h, s, d = 2, 2, 300, 16
    q, k, v, go = (torch.randn(b, h, s, d, generator=g, dtype=torch.float64) for _ in range(4))
    m = torch.rand(b, h, 3, 3, generator=g) > 0.4
    m[:, :, 1, :] = False  # rows 128..255 see no key: O = 0, LSE = -inf
    o, lse = attention_forward(q, k, v, causal=causal, block_mask=m)
    keep = block_keep(m, b, h, s, s)
    if causal:
        keep = keep & torch.ones(s, s, dtype=torch.bool).tril()
    o_d, lse_d = _dense(q, k, v, keep)
    assert torch.allclose(o, o_d, atol=1e-12)
    assert torch.equal(torch.isfinite(lse), torch.isfinite(lse_d))
    assert torch.isneginf(lse[:, :, 128:256]).all() and (o[:, :, 128:256] == 0).all()
    fin = torch.isfinite(lse)
    assert torch.allclose(lse[fin], lse_d[fin], atol=1e-12)
    # Backward: gradients of the dense masked form by autograd.
    qa, ka, va = (t.clone().requires_grad_(True) for t in (q, k, v))
    o_a, _ = _dense(qa, ka, va, keep)
    o_a.backward(go)
    dq, dk, dv = attention_backward(q, k, v, go, causal=causal, block_mask=m)
    for x, y in ((dq, qa.grad), (dk, ka.grad), (dv, va.grad)):
        assert torch.allclose(x, y, atol=1e-10)


def test_all_on_block_mask_changes_nothing():
    g = torch.Generator().manual_seed(4)
    q, k, v = (torch.randn(1, 2, 140, 8, generator=g, dtype=torch.float64) for _ in range(3))
    o, lse = attention_forward(q, k, v, causal=True, sliding_window=20)
    o_m, lse_m = attention_forward(q, k, v, causal=True, sliding_window=20,
                                   block_mask=torch.ones(2, 2, dtype=torch.bool))
    assert torch.equal(o, o_m) and torch.equal(lse, lse_m)
