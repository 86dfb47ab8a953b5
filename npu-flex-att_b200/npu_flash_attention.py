"""B200 flash attention with the operator surface of npu_flash_attention.py.

Drop-in replacement for dropletzhu/npu-flex-att's ``npu_flash_attention``
module: the same function names, arguments, defaults, return values, layouts
([B, H, S, D]) and errors. Every call runs hand-written sm_100a CUDA kernels
through the C ABI of ``libbfa.so`` (include/bfa.h); there is no Triton, no
multi-backend dispatch and no CPU fallback.

Reference map (file:line in npu_flash_attention.py):
  npu_flash_attention_forward   :606-656
  npu_flash_attention_backward  :659-739
  NPUFlexAttention              :742-781
  npu_flex_attention            :784-794
  AttentionConfig               :820-844
  flex_attention                :847-886

Differences that are deliberate:
  * ``block_m`` / ``block_n`` are accepted for compatibility and ignored; the
    kernels pick their own tiles (128 x 128 on the tcgen05 path).
  * The backward honours ``alibi_slope`` and returns the true gradient of the
    forward (the reference backward drops the slopes, :663, :696-732).
  * Key columns past the key length never enter the softmax (the reference's
    non-causal path lets zero-padded keys in, :98, :125).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Optional

import torch

import bfa_lib as _bfa

__all__ = [
    "npu_flash_attention_forward",
    "npu_flash_attention_backward",
    "NPUFlexAttention",
    "npu_flex_attention",
    "AttentionConfig",
    "flex_attention",
    "check_device_status",
]

_CHECK_STATUS = os.environ.get("BFA_CHECK_STATUS", "0") == "1"


def _fast_layout(t: torch.Tensor) -> torch.Tensor:
    """Give 16-bit tensors a layout the TMA path can read (unit inner stride,
    16-byte aligned outer strides); other tensors pass through unchanged and
    the library's generic CUDA kernels handle their strides."""
    if t.dtype not in (torch.float16, torch.bfloat16):
        return t
    ok = (t.stride(-1) == 1 and t.data_ptr() % 16 == 0
          and all(s > 0 and (s * 2) % 16 == 0 for s in t.stride()[:-1]))
    return t if ok else t.contiguous()


def _documents(cu_seqlens, positions: int, device):
    """Per-position document bounds from cumulative document lengths.

    ``cu_seqlens`` (ints, non-decreasing, first 0) cuts the absolute positions
    [0, cu_seqlens[-1]) into documents [cu_seqlens[d], cu_seqlens[d+1]). Returns
    int32 device tensors (start, end) of the document holding each position;
    they must cover every query and key position of the call."""
    if cu_seqlens is None:
        return None
    cu = torch.as_tensor(cu_seqlens).to(device=device, dtype=torch.int64).reshape(-1)
    if cu.numel() < 2 or int(cu[0]) != 0 or bool((cu[1:] < cu[:-1]).any()):
        raise ValueError("cu_seqlens must start at 0 and be non-decreasing")
    total = int(cu[-1])
    if total < positions:
        raise ValueError(f"cu_seqlens covers {total} positions, the call needs {positions}")
    if total >= 2 ** 31:
        raise ValueError("cu_seqlens must stay below 2**31 positions")
    pos = torch.arange(total, device=device, dtype=torch.int64)
    idx = torch.searchsorted(cu, pos, right=True) - 1
    return cu[idx].to(torch.int32).contiguous(), cu[idx + 1].to(torch.int32).contiguous()


BLOCK = 128  # block-sparse mask granularity: 128 query rows x 128 keys


def _block_mask(block_mask, B: int, Hq: int, Sq: int, Sk: int, device):
    """Validated block-sparse mask as a uint8 device tensor of shape
    [B, Hq, ceil(Sq/128), ceil(Sk/128)], batch and head dims possibly broadcast
    (stride 0). Accepts bool or integer tensors of shape [nq, nk], [Hq, nq, nk]
    or [B or 1, Hq or 1, nq, nk]; nonzero means the block is computed. The
    tensor must stay alive until the call's kernels have run (the functions
    below keep it referenced for the call)."""
    if block_mask is None:
        return None
    m = torch.as_tensor(block_mask)
    nq, nk = -(-Sq // BLOCK), -(-Sk // BLOCK)
    while m.dim() < 4:
        m = m.unsqueeze(0)
    if m.dim() != 4 or tuple(m.shape[2:]) != (nq, nk) or m.shape[0] not in (1, B) or m.shape[1] not in (1, Hq):
        raise ValueError(f"block_mask must have shape [B|1, Hq|1, {nq}, {nk}] "
                         f"(128x128 blocks of a {Sq}x{Sk} score matrix), got {tuple(torch.as_tensor(block_mask).shape)}")
    m = (m != 0).to(device=device, dtype=torch.uint8)
    m = m.expand(B, Hq, nq, nk)
    if m.stride(3) != 1:
        m = m.contiguous()
    return m


def _problem(query, key, causal, sliding_window, alibi, scale, soft_cap, q_pos=0, k_pos=0,
             docs=None, blk=None):
    B, Hq, Sq, D = query.shape
    _, Hkv, Sk, _ = key.shape
    pr = _bfa.Problem()
    pr.batch, pr.heads_q, pr.heads_kv = B, Hq, Hkv
    pr.seqlen_q, pr.seqlen_k, pr.head_dim = Sq, Sk, D
    pr.dtype = _bfa.bfa_dtype(query.dtype)
    pr.causal = 1 if causal else 0
    pr.sliding_window = int(sliding_window)
    pr.scale = float(scale)
    pr.soft_cap = float(soft_cap)
    pr.alibi_slopes = alibi.data_ptr() if alibi is not None else None
    pr.q_pos_offset, pr.k_pos_offset = int(q_pos), int(k_pos)
    if docs is not None:
        pr.doc_start, pr.doc_end = docs[0].data_ptr(), docs[1].data_ptr()
    if blk is not None:
        pr.block_mask = blk.data_ptr()
        for d in range(3):
            pr.block_mask_stride[d] = blk.stride(d)
    return pr


def _alibi(alibi_slope, hq: int, device) -> Optional[torch.Tensor]:
    if alibi_slope is None:
        return None
    a = torch.as_tensor(alibi_slope, dtype=torch.float32).to(device).reshape(-1).contiguous()
    if a.numel() != hq:
        raise RuntimeError(f"alibi_slope must have one slope per query head ({hq}), got {a.numel()}")
    return a


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("npu_flash_attention (B200 build) needs CUDA tensors; "
                               "there is no CPU path")


def _after_call(device):
    if _CHECK_STATUS:
        check_device_status(device)


def check_device_status(device=None) -> None:
    """Synchronise and raise if a kernel on `device` reported a device-side
    timeout since the last check (then clear the report)."""
    device = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    code = _bfa.read_and_clear_status(device)
    if code != 0:
        _bfa.check(code)


def npu_flash_attention_forward(
    query, key, value,
    causal=False,
    sliding_window=0,
    alibi_slope=None,
    scale=None,
    block_m=16,
    block_n=64,
    return_lse=False,
    soft_cap=0.0,
    *,
    q_pos_offset=0,
    k_pos_offset=0,
    cu_seqlens=None,
    block_mask=None,
    _wait_timeout_ns=0,
    _debug_flags=0,
    _merge_into=None,
):
    """Attention forward: O (and the fp32 natural-log LSE when `return_lse`).

    Mirrors npu_flash_attention.py:606-656. Keyword-only extras (not in the
    reference): absolute position offsets for context-parallel shards, and
    document masking -- ``cu_seqlens`` (cumulative document lengths over the
    absolute positions, first 0) keeps only pairs inside one document, on
    top of the other masks (packed variable-length sequences) -- and a
    block-sparse mask: ``block_mask`` (bool/int, [B|1, Hq|1, ceil(Sq/128),
    ceil(Sk/128)]) computes only the 128x128 blocks of the score matrix it
    marks, again on top of the other masks; the kernels skip the other
    blocks. Rows left with no key give O = 0 and LSE = -inf.

    ``_merge_into`` (internal: the context-parallel ring) is a pair (O_acc
    fp32 [B, Hq, Sq, D], LSE_acc fp32 contiguous [B, Hq, Sq]) holding a
    running result; the call merges its own result into both in place (the
    library's epilogue merge, bfa_fwd_args.accumulate) and returns them.
    """
    B, Hq, Sq, D = query.shape
    Bk, Hkv, Sk, Dk = key.shape
    Bv, Hkv2, Sv, Dv = value.shape
    assert D == Dk, "Q and K head dims must match"
    assert Dv == D, "V head dim must match Q head dim for this kernel"
    assert Hq % Hkv == 0, "Hq must be divisible by Hkv"
    _require_cuda(query, key, value)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dev = query.device
    alibi = _alibi(alibi_slope, Hq, dev)
    q, k, v = _fast_layout(query), _fast_layout(key), _fast_layout(value)
    if _merge_into is not None:
        O, LSE = _merge_into
        if (O.dtype != torch.float32 or tuple(O.shape) != (B, Hq, Sq, D) or O.device != dev
                or LSE.dtype != torch.float32 or tuple(LSE.shape) != (B, Hq, Sq)
                or LSE.device != dev or not LSE.is_contiguous()):
            raise ValueError("_merge_into takes fp32 O [B, Hq, Sq, D] and contiguous fp32 LSE "
                             "[B, Hq, Sq] on the query's device")
        o_k = O
    else:
        O = torch.empty_like(query)
        o_k = _fast_layout(O) if O.data_ptr() else O
        LSE = torch.empty(B, Hq, Sq, device=dev, dtype=torch.float32)
    lib = _bfa.load()
    docs = _documents(cu_seqlens, max(q_pos_offset + Sq, k_pos_offset + Sk), dev)
    blk = _block_mask(block_mask, B, Hq, Sq, Sk, dev)
    pr = _problem(q, k, causal, sliding_window, alibi, scale, soft_cap, q_pos_offset, k_pos_offset, docs,
                  blk)
    args = _bfa.FwdArgs()
    args.q, args.k, args.v, args.o = _bfa.tensor(q), _bfa.tensor(k), _bfa.tensor(v), _bfa.tensor(o_k)
    args.lse = LSE.data_ptr()
    args.status = _bfa.status_word(dev).data_ptr()
    args.wait_timeout_ns = int(_wait_timeout_ns)
    args.debug_flags = int(_debug_flags)
    args.accumulate = 1 if _merge_into is not None else 0
    with torch.cuda.device(dev):
        # Scratch of the split-KV decoding path (few query rows per KV head),
        # from torch's caching allocator: the library allocates nothing. A
        # merging call never takes that path.
        ws_bytes = 0 if _merge_into is not None else lib.bfa_fwd_workspace_bytes(pr)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
        if ws is not None:
            args.workspace, args.workspace_bytes = ws.data_ptr(), ws_bytes
        _bfa.check(lib.bfa_fwd(pr, args, _bfa.stream_ptr(dev)))
    if o_k is not O:
        O.copy_(o_k)
    _after_call(dev)
    if return_lse:
        return O, LSE
    return O


def npu_flash_attention_backward(
    query, key, value, out, lse, grad_out,
    causal=False,
    sliding_window=0,
    alibi_slope=None,
    scale=None,
    block_m=16,
    block_n=32,
    soft_cap=0.0,
    *,
    q_pos_offset=0,
    k_pos_offset=0,
    cu_seqlens=None,
    block_mask=None,
    _wait_timeout_ns=0,
    _debug_flags=0,
    _phases=0,
    _workspace=None,
    _outputs=None,
    _accumulate=False,
):
    """Attention backward: (dQ, dK, dV), dK/dV summed over each GQA group.

    ``_phases`` / ``_workspace`` / ``_outputs`` (internal) let a benchmark
    launch Δ, dK/dV and dQ as separate calls on one workspace and reuse the
    gradient buffers, so each kernel can be timed on its own.
    ``_accumulate`` (internal) adds the gradients into ``_outputs``, which must
    then be fp32: a blockwise (context-parallel) backward sums its partial
    gradients without rounding each one to 16 bits.

    Mirrors npu_flash_attention.py:659-739; Δ, both gradient kernels and the
    GQA reduction run on the device in one library call.
    """
    B, Hq, Sq, D = query.shape
    Bk, Hkv, Sk, Dk = key.shape
    assert D == Dk, "Q and K head dims must match"
    assert Hq % Hkv == 0, "Hq must be divisible by Hkv"
    assert out is not None, "backward requires forward output `out` to compute Delta"
    _require_cuda(query, key, value, out, lse, grad_out)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dev = query.device
    alibi = _alibi(alibi_slope, Hq, dev)
    q, k, v = _fast_layout(query), _fast_layout(key), _fast_layout(value)
    o, do = _fast_layout(out), _fast_layout(grad_out.to(query.dtype))
    lse_c = lse.to(torch.float32).contiguous()
    if _outputs is not None:
        DQ, DK, DV = _outputs
        if _accumulate and not all(t.dtype == torch.float32 for t in _outputs):
            raise ValueError("_accumulate needs fp32 gradient buffers")
    elif _accumulate:
        raise ValueError("_accumulate needs _outputs")
    else:
        DQ = torch.empty_like(query)
        DK = torch.empty(B, Hkv, Sk, D, device=dev, dtype=key.dtype)
        DV = torch.empty(B, Hkv, Sk, D, device=dev, dtype=value.dtype)
    dq_k = _fast_layout(DQ) if DQ.data_ptr() else DQ
    lib = _bfa.load()
    docs = _documents(cu_seqlens, max(q_pos_offset + Sq, k_pos_offset + Sk), dev)
    blk = _block_mask(block_mask, B, Hq, Sq, Sk, dev)
    pr = _problem(q, k, causal, sliding_window, alibi, scale, soft_cap, q_pos_offset, k_pos_offset, docs,
                  blk)
    args = _bfa.BwdArgs()
    args.q, args.k, args.v = _bfa.tensor(q), _bfa.tensor(k), _bfa.tensor(v)
    args.o, args.dout = _bfa.tensor(o), _bfa.tensor(do)
    args.lse = lse_c.data_ptr()
    args.dq, args.dk, args.dv = _bfa.tensor(dq_k), _bfa.tensor(DK), _bfa.tensor(DV)
    args.status = _bfa.status_word(dev).data_ptr()
    args.wait_timeout_ns = int(_wait_timeout_ns)
    args.debug_flags = int(_debug_flags)
    args.phases = int(_phases)
    args.accumulate = 1 if _accumulate else 0
    ws_bytes = lib.bfa_bwd_workspace_bytes(pr)
    ws = _workspace if _workspace is not None else torch.empty(
        max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    assert ws.numel() >= ws_bytes
    with torch.cuda.device(dev):
        _bfa.check(lib.bfa_bwd(pr, args, ws.data_ptr(), ws_bytes, _bfa.stream_ptr(dev)))
    if dq_k is not DQ:
        DQ.copy_(dq_k)
    _after_call(dev)
    return DQ, DK, DV


class NPUFlexAttention(torch.autograd.Function):
    """torch.autograd.Function over the two library calls: forward saves
    (q, k, v, LSE, O) for the backward, which returns gradients for q, k and
    v only (the mask arguments get None). Same class name, argument order and
    saved state as the reference's autograd class
    (npu_flash_attention.py:742-781), so code that calls ``.apply`` on it
    keeps working; two optional arguments are appended, ``cu_seqlens`` and
    ``block_mask`` (document and block-sparse masking, see
    npu_flash_attention_forward)."""

    @staticmethod
    def forward(ctx, query, key, value, causal=False, sliding_window=0,
                alibi_slope=None, scale=None, block_m=16, block_n=64, soft_cap=0.0,
                cu_seqlens=None, block_mask=None):
        ctx.cu_seqlens = cu_seqlens
        ctx.block_mask = block_mask
        ctx.causal = causal
        ctx.sliding_window = sliding_window
        ctx.alibi_slope = alibi_slope
        ctx.scale = scale
        ctx.block_m = block_m
        ctx.block_n = block_n
        ctx.soft_cap = soft_cap
        with torch.no_grad():
            out, lse = npu_flash_attention_forward(
                query, key, value,
                causal=causal, sliding_window=sliding_window,
                alibi_slope=alibi_slope, scale=scale,
                block_m=block_m, block_n=block_n, return_lse=True,
                soft_cap=soft_cap, cu_seqlens=cu_seqlens, block_mask=block_mask,
            )
        ctx.save_for_backward(query, key, value, lse, out)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        query, key, value, lse, out = ctx.saved_tensors
        DQ, DK, DV = npu_flash_attention_backward(
            query, key, value, out, lse, grad_out,
            causal=ctx.causal, sliding_window=ctx.sliding_window,
            alibi_slope=ctx.alibi_slope, scale=ctx.scale,
            block_m=ctx.block_m, block_n=ctx.block_n,
            soft_cap=ctx.soft_cap, cu_seqlens=ctx.cu_seqlens, block_mask=ctx.block_mask,
        )
        return DQ, DK, DV, None, None, None, None, None, None, None, None, None


def npu_flex_attention(
    query, key, value,
    causal=False, sliding_window=0,
    alibi_slope=None, scale=None,
    block_m=16, block_n=64,
    soft_cap=0.0,
    cu_seqlens=None,
    block_mask=None,
):
    """Functional form of NPUFlexAttention.apply with keyword defaults
    (signature of npu_flash_attention.py:784-794, plus ``cu_seqlens`` and
    ``block_mask``)."""
    return NPUFlexAttention.apply(
        query, key, value, causal, sliding_window,
        alibi_slope, scale, block_m, block_n, soft_cap, cu_seqlens, block_mask,
    )


@dataclass
class AttentionConfig:
    """Bundle of the mask and logit options that flex_attention applies
    (fields, defaults and validation of npu_flash_attention.py:820-844).

    A negative window or cap raises ValueError when the config is built.
    For instance a local-attention layer with capped logits:
        cfg = AttentionConfig(causal=True, sliding_window=4096, soft_cap=50.0)
        o = flex_attention(q, k, v, config=cfg)
    ``cu_seqlens`` (appended after the reference's fields) adds document
    masking over packed sequences:
        cfg = AttentionConfig(causal=True, cu_seqlens=torch.tensor([0, 700, 1024]))
    and ``block_mask`` a block-sparse mask (128x128 blocks of the score
    matrix, see npu_flash_attention_forward).
    """
    causal: bool = False
    sliding_window: int = 0
    alibi_slope: Optional[torch.Tensor] = None
    scale: Optional[float] = None
    soft_cap: float = 0.0
    block_m: int = 16
    block_n: int = 64
    cu_seqlens: Optional[torch.Tensor] = None
    block_mask: Optional[torch.Tensor] = None

    def __post_init__(self):
        if self.sliding_window < 0:
            raise ValueError("sliding_window must be >= 0")
        if self.soft_cap < 0:
            raise ValueError("soft_cap must be >= 0")


def flex_attention(query, key, value, config: Optional[AttentionConfig] = None, **kwargs):
    """Differentiable attention driven by an AttentionConfig. With no
    ``config`` the keyword arguments build one; with a config they are not
    looked at (the rule of npu_flash_attention.py:847-886)."""
    if config is None:
        config = AttentionConfig(**kwargs)
    return npu_flex_attention(
        query, key, value,
        causal=config.causal,
        sliding_window=config.sliding_window,
        alibi_slope=config.alibi_slope,
        scale=config.scale,
        block_m=config.block_m,
        block_n=config.block_n,
        soft_cap=config.soft_cap,
        cu_seqlens=config.cu_seqlens,
        block_mask=config.block_mask,
    )
