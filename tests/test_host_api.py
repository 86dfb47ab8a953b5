"""Host-side behaviour of the drop-in module (CPU only, no kernels run).

Mirrors the reference's argument handling: AttentionConfig validation
(npu_flash_attention.py:840-844), flex_attention's config/kwargs rule
(:875-876) and the shape assertions (:620-622, tested by
test/test_real_world.py:65-85).
"""
import inspect

import pytest
import torch

import npu_flash_attention as nfa


def test_attention_config_validation():
    with pytest.raises(ValueError):
        nfa.AttentionConfig(sliding_window=-1)
    with pytest.raises(ValueError):
        nfa.AttentionConfig(soft_cap=-0.5)
    cfg = nfa.AttentionConfig(causal=True, sliding_window=1024, soft_cap=50.0)
    assert (cfg.causal, cfg.sliding_window, cfg.soft_cap, cfg.block_m, cfg.block_n) == (True, 1024, 50.0, 16, 64)


def test_signatures_match_reference():
    sig = inspect.signature(nfa.npu_flash_attention_forward)
    names = list(sig.parameters)[:11]
    assert names == ["query", "key", "value", "causal", "sliding_window", "alibi_slope",
                     "scale", "block_m", "block_n", "return_lse", "soft_cap"]
    assert sig.parameters["block_m"].default == 16 and sig.parameters["block_n"].default == 64
    sig = inspect.signature(nfa.npu_flash_attention_backward)
    names = list(sig.parameters)[:13]
    assert names == ["query", "key", "value", "out", "lse", "grad_out", "causal",
                     "sliding_window", "alibi_slope", "scale", "block_m", "block_n", "soft_cap"]
    assert sig.parameters["block_n"].default == 32
    sig = inspect.signature(nfa.npu_flex_attention)
    # The reference's ten parameters in order, then this build's document and
    # block-sparse masks.
    assert list(sig.parameters) == ["query", "key", "value", "causal", "sliding_window",
                                    "alibi_slope", "scale", "block_m", "block_n", "soft_cap",
                                    "cu_seqlens", "block_mask"]
    assert sig.parameters["cu_seqlens"].default is None
    assert sig.parameters["block_mask"].default is None


def test_block_mask_validation_and_broadcast():
    m = nfa._block_mask(torch.tensor([[1, 0], [1, 1]], dtype=torch.bool), 2, 4, 200, 129, "cpu")
    assert m.shape == (2, 4, 2, 2) and m.dtype == torch.uint8
    assert m.stride(0) == 0 and m.stride(1) == 0 and m.stride(3) == 1
    assert m[1, 3].tolist() == [[1, 0], [1, 1]]
    m = nfa._block_mask(torch.ones(4, 1, 1, dtype=torch.int32), 2, 4, 100, 100, "cpu")
    assert m.shape == (2, 4, 1, 1) and m.stride(0) == 0 and m.stride(1) == 1
    with pytest.raises(ValueError):
        nfa._block_mask(torch.ones(2, 3), 1, 1, 256, 256, "cpu")
    with pytest.raises(ValueError):
        nfa._block_mask(torch.ones(3, 4, 2, 2), 2, 4, 256, 256, "cpu")
    assert nfa._block_mask(None, 1, 1, 1, 1, "cpu") is None


def test_shape_assertions_fire_before_device_work():
    q = torch.randn(1, 1, 8, 64)
    with pytest.raises(AssertionError):
        nfa.npu_flash_attention_forward(q, torch.randn(1, 1, 8, 128), torch.randn(1, 1, 8, 64))
    with pytest.raises(AssertionError):
        nfa.npu_flash_attention_forward(torch.randn(1, 3, 8, 64), torch.randn(1, 2, 8, 64),
                                        torch.randn(1, 2, 8, 64))
    with pytest.raises(AssertionError):
        nfa.npu_flash_attention_forward(q, q, torch.randn(1, 1, 8, 32))
    with pytest.raises(AssertionError):
        nfa.npu_flash_attention_backward(q, q, q, None, torch.zeros(1, 1, 8), q)


def test_cpu_tensors_are_refused_not_computed():
    q = torch.randn(1, 1, 8, 64)
    with pytest.raises(RuntimeError, match="no CPU path"):
        nfa.npu_flash_attention_forward(q, q, q)


def test_flex_attention_ignores_kwargs_when_config_given(monkeypatch):
    seen = {}

    def fake(query, key, value, **kw):
        seen.update(kw)
        return query
    monkeypatch.setattr(nfa, "npu_flex_attention", fake)
    cfg = nfa.AttentionConfig(causal=True, soft_cap=3.0)
    nfa.flex_attention(torch.zeros(1), torch.zeros(1), torch.zeros(1), config=cfg, causal=False)
    assert seen["causal"] is True and seen["soft_cap"] == 3.0
    nfa.flex_attention(torch.zeros(1), torch.zeros(1), torch.zeros(1), sliding_window=7)
    assert seen["sliding_window"] == 7 and seen["causal"] is False
    with pytest.raises(ValueError):
        nfa.flex_attention(torch.zeros(1), torch.zeros(1), torch.zeros(1), sliding_window=-2)
