"""CPU restatement of the reference attention math -- TEST INFRASTRUCTURE ONLY.

This module is the parity oracle. Only ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and
only as the checker or as the timed CPU baseline. The product path
(``npu_flash_attention``) never calls it and has no CPU fallback.

It restates, in float64 (or float32) torch-on-CPU arithmetic, what
``npu_flash_attention.py`` of dropletzhu/npu-flex-att computes:

* forward  -- ``flash_attn_fwd_kernel``        npu_flash_attention.py:17-166
* dQ       -- ``flash_attn_bwd_dq_kernel``     npu_flash_attention.py:298-402
* dK/dV    -- ``flash_attn_bwd_dkdv_kernel``   npu_flash_attention.py:407-560
* host Δ   -- ``(out*grad_out).sum(-1)``       npu_flash_attention.py:685
* GQA sum  -- ``DK.view(B,Hkv,G,Sk,D).sum(2)``  npu_flash_attention.py:735-737

Semantics (each cites the reference line it follows):

1. logits ``s = (q·kᵀ)·scale``                                  (:102)
2. soft-cap ``s = cap·tanh(s/cap)`` when cap > 0, before ALiBi   (:105-106)
3. ALiBi    ``s += slope[hq]·(i − j)`` (positive sign, q-head)   (:108-109)
4. causal   keep ``i ≥ j`` in local indices, top-left aligned    (:78, :139)
5. window   keep ``i − j ≤ W`` (W+1 keys incl. the diagonal)     (:70-71, :141)
6. softmax over the kept keys; ``lse`` = natural-log logsumexp   (:111-118, :161)
7. GQA      ``hkv = hq // (Hq/Hkv)``; dK/dV summed over the group (:42, :735-737)
8. backward ``dP = dO·Vᵀ``, ``Δ = rowsum(O∘dO)``, ``dS = P∘(dP − Δ)``,
   chained through ``1 − tanh²`` and ``scale``                    (:386-399, :502-516, :685)

Where this oracle deliberately differs from the reference kernels:

* Key columns ``j ≥ Sk`` do not exist here. The reference loads padded K rows
  as zeros and, in its non-causal path, keeps their logit 0 (npu_flash_attention.py:98,125;
  its README lists it as a known bug). The math path has no padding, so it has no
  such columns.
* ALiBi gradients: the reference backward never receives the slopes
  (npu_flash_attention.py:663, not forwarded at :696-732), so its dQ/dK/dV are not the
  gradient of its own forward. ``attention_backward`` defaults to the true
  gradient (``alibi_in_backward=True``). With ``alibi_in_backward=False`` it
  reproduces the reference kernels' behaviour, which the golden-vector tests
  use to pin the rest of the backward math.
* Fully masked rows (possible with a non-causal window when ``i − W ≥ Sk``)
  give ``O = 0`` and ``lse = -inf`` and zero gradients. The reference gives the
  same O/LSE when the row's tiles are all skipped.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

__all__ = [
    "MaskSpec",
    "keep_mask",
    "logits",
    "attention_forward",
    "attention_backward",
    "unmasked_pairs",
    "attention_flops",
]


@dataclass(frozen=True)
class MaskSpec:
    causal: bool = False
    sliding_window: int = 0
    soft_cap: float = 0.0
    scale: Optional[float] = None
    q_offset: int = 0
    k_offset: int = 0


def keep_mask(sq: int, sk: int, causal: bool, window: int,
              q_offset: int = 0, k_offset: int = 0, cu_seqlens=None) -> torch.Tensor:
    """Boolean [Sq, Sk] keep-mask (npu_flash_attention.py:139,141).

    ``q_offset``/``k_offset`` shift the row/column positions (context-parallel
    shards); both are 0 for the reference's own calls. ``cu_seqlens``
    (cumulative document lengths over absolute positions, first 0) adds
    document masking, which the reference does not have (its README lists
    document / block masks as missing): a pair is kept only when i and j lie
    in the same document [cu[d], cu[d+1]).
    """
    i = torch.arange(sq).view(-1, 1) + q_offset
    j = torch.arange(sk).view(1, -1) + k_offset
    keep = torch.ones(sq, sk, dtype=torch.bool)
    if causal:
        keep &= i >= j
    if window > 0:
        keep &= (i - j) <= window
    if cu_seqlens is not None:
        cu = torch.as_tensor(cu_seqlens, dtype=torch.int64).cpu().reshape(-1)
        doc_i = torch.searchsorted(cu, i.reshape(-1), right=True).view(-1, 1)
        doc_j = torch.searchsorted(cu, j.reshape(-1), right=True).view(1, -1)
        keep &= doc_i == doc_j
    return keep


def block_keep(block_mask, b: int, hq: int, sq: int, sk: int, block: int = 128) -> torch.Tensor:
    """Element keep-mask [B, Hq, Sq, Sk] of a block-sparse mask: pair (i, j) of
    (b, h) is kept when block (i // 128, j // 128) is nonzero; ``block_mask``
    is [nq, nk], [Hq, nq, nk] or [B|1, Hq|1, nq, nk] over the call's own row
    and key indices. The reference has no block masks (its README lists them
    as missing); this restates the rule the build adds."""
    m = torch.as_tensor(block_mask).cpu() != 0
    while m.dim() < 4:
        m = m.unsqueeze(0)
    m = m.expand(b, hq, m.shape[2], m.shape[3])
    m = m.repeat_interleave(block, dim=2).repeat_interleave(block, dim=3)
    return m[:, :, :sq, :sk]


def _expand_kv(x: torch.Tensor, hq: int) -> torch.Tensor:
    """GQA head map hkv = hq // G (npu_flash_attention.py:42), as repeat_interleave."""
    hkv = x.shape[1]
    g = hq // hkv
    return x.repeat_interleave(g, dim=1) if g > 1 else x


def logits(q, k, *, scale, soft_cap=0.0, alibi_slope=None,
           q_offset=0, k_offset=0):
    """Un-masked logits ``u`` and the tanh value (for the soft-cap chain).

    Returns ``(u, t)`` where ``t = tanh(s/cap)`` or ``None``.
    Follows npu_flash_attention.py:102-109.
    """
    hq = q.shape[1]
    kx = _expand_kv(k, hq)
    s = torch.matmul(q, kx.transpose(-2, -1)) * scale
    t = None
    if soft_cap > 0.0:
        t = torch.tanh(s / soft_cap)
        s = t * soft_cap
    if alibi_slope is not None:
        sq, sk = q.shape[2], k.shape[2]
        i = torch.arange(sq, dtype=s.dtype).view(-1, 1) + q_offset
        j = torch.arange(sk, dtype=s.dtype).view(1, -1) + k_offset
        slope = alibi_slope.to(s.dtype).view(1, hq, 1, 1)
        s = s + slope * (i - j)
    return s, t


def attention_forward(q, k, v, *, causal=False, sliding_window=0,
                      alibi_slope=None, scale=None, soft_cap=0.0,
                      q_offset=0, k_offset=0, cu_seqlens=None, block_mask=None,
                      dtype=torch.float64):
    """Forward oracle: returns ``(O, LSE)`` in ``dtype`` (O) and ``dtype`` (LSE).

    npu_flash_attention.py:17-166 (kernel) and :606-656 (host wrapper:
    ``scale=None`` -> 1/sqrt(D) at :625-626).
    """
    d = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    qf, kf, vf = q.to(dtype), k.to(dtype), v.to(dtype)
    slope = None if alibi_slope is None else alibi_slope.to(dtype).cpu()
    u, _ = logits(qf, kf, scale=scale, soft_cap=soft_cap, alibi_slope=slope,
                  q_offset=q_offset, k_offset=k_offset)
    keep = keep_mask(q.shape[2], k.shape[2], causal, sliding_window,
                     q_offset, k_offset, cu_seqlens)
    if block_mask is not None:
        keep = keep & block_keep(block_mask, q.shape[0], q.shape[1], q.shape[2], k.shape[2])
    u = u.masked_fill(~keep, float("-inf"))
    lse = torch.logsumexp(u, dim=-1)
    finite = torch.isfinite(lse)
    p = torch.exp(u - torch.where(finite, lse, torch.zeros_like(lse)).unsqueeze(-1))
    p = torch.where(finite.unsqueeze(-1), p, torch.zeros_like(p))
    o = torch.matmul(p, _expand_kv(vf, q.shape[1]))
    return o, lse


def attention_backward(q, k, v, grad_out, *, causal=False, sliding_window=0,
                       alibi_slope=None, scale=None, soft_cap=0.0,
                       q_offset=0, k_offset=0, alibi_in_backward=True,
                       out=None, lse=None, dtype=torch.float64,
                       operand_dtype=None, cu_seqlens=None, block_mask=None):
    """Backward oracle: returns ``(dQ, dK, dV)`` with dK/dV per KV head.

    Restates npu_flash_attention.py:659-739 and the two kernels :298-560.
    ``out``/``lse`` default to this oracle's own forward. ``Δ`` is
    ``rowsum(out∘grad_out)`` (:685). With ``alibi_in_backward=False`` the
    probabilities are recomputed without the ALiBi bias against the given
    ``lse``, exactly as the reference kernels do.

    ``operand_dtype`` (fp16/bf16) rounds P and dS to that type before they
    enter the dV, dK and dQ products, as the reference kernels do
    (``p.to(v.dtype)`` :506/:545, ``ds.to(k.dtype)`` :516/:555,
    ``ds.to(q.dtype)`` :399); the products themselves stay in ``dtype``.
    """
    d = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    hq, hkv = q.shape[1], k.shape[1]
    g = hq // hkv
    qf, kf, vf, dof = (x.to(dtype) for x in (q, k, v, grad_out))
    slope = None if alibi_slope is None else alibi_slope.to(dtype).cpu()
    if out is None or lse is None:
        o_ref, lse_ref = attention_forward(
            q, k, v, causal=causal, sliding_window=sliding_window,
            alibi_slope=alibi_slope, scale=scale, soft_cap=soft_cap,
            q_offset=q_offset, k_offset=k_offset, cu_seqlens=cu_seqlens,
            block_mask=block_mask, dtype=dtype)
        out = o_ref if out is None else out
        lse = lse_ref if lse is None else lse
    of, lsef = out.to(dtype), lse.to(dtype)
    u, t = logits(qf, kf, scale=scale, soft_cap=soft_cap,
                  alibi_slope=slope if alibi_in_backward else None,
                  q_offset=q_offset, k_offset=k_offset)
    keep = keep_mask(q.shape[2], k.shape[2], causal, sliding_window,
                     q_offset, k_offset, cu_seqlens)
    if block_mask is not None:
        keep = keep & block_keep(block_mask, q.shape[0], q.shape[1], q.shape[2], k.shape[2])
    finite = torch.isfinite(lsef).unsqueeze(-1)
    p = torch.exp(u - torch.where(finite, lsef.unsqueeze(-1), torch.zeros_like(u[..., :1])))
    p = torch.where(keep & finite, p, torch.zeros_like(p))
    vx = _expand_kv(vf, hq)
    kx = _expand_kv(kf, hq)
    dp = torch.matmul(dof, vx.transpose(-2, -1))
    delta = (of * dof).sum(-1, keepdim=True)
    ds = p * (dp - delta)
    if t is not None:
        ds = ds * (1.0 - t * t)
    ds = ds * scale
    if operand_dtype is not None:
        p = p.to(operand_dtype).to(dtype)
        ds = ds.to(operand_dtype).to(dtype)
    dq = torch.matmul(ds, kx)
    dk_h = torch.matmul(ds.transpose(-2, -1), qf)
    dv_h = torch.matmul(p.transpose(-2, -1), dof)
    b, _, sk, _ = k.shape
    dk = dk_h.view(b, hkv, g, sk, d).sum(2)
    dv = dv_h.view(b, hkv, g, sk, d).sum(2)
    return dq, dk, dv


def reference_backward(q, k, v, grad_out, *, dtype=torch.float64, **mask):
    """Gradients of the operator as a caller sees it: the forward's output is
    rounded to the input dtype before Δ = rowsum(O∘dO) is formed, as the
    autograd wrapper saves the stored ``out`` (npu_flash_attention.py:760, :772-777),
    and P / dS enter the gradient products in the input dtype (16-bit inputs).
    """
    o, lse = attention_forward(q, k, v, dtype=dtype, **mask)
    op = q.dtype if q.dtype in (torch.float16, torch.bfloat16) else None
    return attention_backward(q, k, v, grad_out, out=o.to(q.dtype), lse=lse,
                              dtype=dtype, operand_dtype=op, **mask)


def attention_forward_reference_tiles(q, k, v, *, causal=False, sliding_window=0,
                                      alibi_slope=None, scale=None, soft_cap=0.0,
                                      block_m=16, block_n=64,
                                      dtype=torch.float64):
    """The reference forward INCLUDING its padded-key behaviour (pinning aid).

    Walks the same key tiles as ``flash_attn_fwd_kernel`` (npu_flash_attention.py:65-150):
    per q-block ``start_n = max(pid_m·BM − W, 0)`` when W > 0 (:66-71), a causal
    ``kv_end = min((pid_m+1)·BM, Sk)`` (:77-80), an unmasked prefix up to
    ``full_end`` for pure causal (:88-118) and a masked suffix (:121-150), each
    tile BLOCK_N keys wide. Keys at ``j ≥ Sk`` load as zero K/V rows (:98,125), so
    their logit is ``0`` (+ the ALiBi term) and they are dropped only by the
    masks of the masked suffix. With no such keys visited this equals
    ``attention_forward``; the golden tests use it to pin the cases where the
    reference's padding shows.
    """
    d = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    b, hq, sq, _ = q.shape
    sk = k.shape[2]
    w = sliding_window
    visited = {}
    for pid_m in range((sq + block_m - 1) // block_m):
        start_n = max(pid_m * block_m - w, 0) if w > 0 else 0
        kv_end = min((pid_m + 1) * block_m, sk) if causal else sk
        full_end = (pid_m * block_m // block_n) * block_n if (causal and w == 0) else start_n
        tiles = [(sn, False) for sn in range(start_n, full_end, block_n)]
        tiles += [(sn, True) for sn in range(full_end, kv_end, block_n)]
        visited[pid_m] = tiles
    sk_pad = max([sk] + [sn + block_n for ts in visited.values() for sn, _ in ts])
    pad = sk_pad - sk
    kf, vf = k.to(dtype), v.to(dtype)
    if pad:
        zeros = torch.zeros(b, k.shape[1], pad, d, dtype=dtype)
        kf, vf = torch.cat([kf, zeros], 2), torch.cat([vf, zeros], 2)
    slope = None if alibi_slope is None else alibi_slope.to(dtype).cpu()
    u, _ = logits(q.to(dtype), kf, scale=scale, soft_cap=soft_cap, alibi_slope=slope)
    keep = torch.zeros(sq, sk_pad, dtype=torch.bool)
    for pid_m, tiles in visited.items():
        for i in range(pid_m * block_m, min((pid_m + 1) * block_m, sq)):
            for sn, masked in tiles:
                for j in range(sn, sn + block_n):
                    ok = True
                    if masked and causal:
                        ok &= i >= j
                    if masked and w > 0:
                        ok &= (i - j) <= w
                    keep[i, j] = ok
    u = u.masked_fill(~keep, float("-inf"))
    lse = torch.logsumexp(u, dim=-1)
    finite = torch.isfinite(lse)
    p = torch.exp(u - torch.where(finite, lse, torch.zeros_like(lse)).unsqueeze(-1))
    p = torch.where(finite.unsqueeze(-1), p, torch.zeros_like(p))
    return torch.matmul(p, _expand_kv(vf, hq)), lse


def unmasked_pairs(sq: int, sk: int, causal: bool, window: int,
                   q_offset: int = 0, k_offset: int = 0) -> int:
    """Element-exact count of kept (i, j) pairs for one head (closed form)."""
    total = 0
    for i in range(sq):
        gi = i + q_offset
        lo, hi = k_offset, k_offset + sk - 1
        if causal:
            hi = min(hi, gi)
        if window > 0:
            lo = max(lo, gi - window)
        if hi >= lo:
            total += hi - lo + 1
    return total


def attention_flops(batch: int, heads_q: int, sq: int, sk: int, d: int,
                    causal: bool, window: int, fwd: bool = True,
                    bwd: bool = True) -> float:
    """Algorithmic FLOPs on unmasked pairs: fwd 4·D, bwd 10·D per pair per q-head."""
    pairs = unmasked_pairs(sq, sk, causal, window) * batch * heads_q
    per = (4 * d if fwd else 0) + (10 * d if bwd else 0)
    return float(pairs) * per
