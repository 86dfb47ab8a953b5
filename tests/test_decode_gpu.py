"""GPU parity of the split-KV decoding forward (csrc/decode.cu).

bfa_fwd takes this path when the G q-heads of a KV head have at most 64 query
rows together (G·Sq <= 64; one CTA per group of up to 16 rows). It is the
working form of the reference's unused split-KV forward + reduce
(npu_flash_attention.py:171-293). Each case checks
the decode result against the CPU oracle with the forward tolerances of
test_parity_gpu.py (fp32 1e-4, fp16 1e-2, bf16 2e-2; LSE 1e-3 relative) and
against the regular path run on the same inputs (BFA_FWD_DECODE=0), and that
the decode path really ran (two launches: the split kernel and the merge).
"""
import os

import pytest
import torch

import bfa_lib
import npu_flash_attention as nfa
from oracle.attention_math import attention_forward
from test_parity_gpu import DEV, LSE_RTOL, TOL, _err, _inputs, _lse_err

pytestmark = pytest.mark.gpu

# (b, hq, hkv, sq, sk, d)
SHAPES = [
    (2, 8, 2, 1, 3000, 128),  # G = 4, one query per head, long key sequence
    (1, 16, 2, 2, 4096, 128),  # G = 8, 16 rows: one full row group
    (3, 4, 4, 4, 1000, 64),  # MHA, 4 queries
    (1, 4, 1, 3, 777, 256),  # D = 256, key count not a multiple of the chunk
    (2, 2, 2, 1, 65, 128),  # one full 64-key chunk + 1 key
    (1, 32, 4, 4, 2048, 128),  # G = 8, 4 queries: 32 rows, two row groups
    (1, 8, 1, 5, 999, 128),  # G = 8, 5 queries: 40 rows, a ragged third row group
    (2, 16, 2, 8, 1500, 64),  # G = 8, 8 queries: 64 rows, the limit (four row groups)
]

MASKS = {
    "none": {},
    "causal": {"causal": True},
    # The decoding mask: the queries are the last Sq positions of the keys.
    "causal_end": {"causal": True, "end_aligned": True},
    "window_end": {"causal": True, "sliding_window": 700, "end_aligned": True},
    "window": {"sliding_window": 100},
    "softcap": {"soft_cap": 30.0},
    "alibi": {"alibi": True},
    "scale": {"scale": 0.3},
}


def _run(q, k, v, kw, decode):
    prev = os.environ.get("BFA_FWD_DECODE")
    if decode:
        os.environ.pop("BFA_FWD_DECODE", None)
    else:
        os.environ["BFA_FWD_DECODE"] = "0"
    try:
        lib = bfa_lib.load()
        n0 = lib.bfa_launch_count()
        o, lse = nfa.npu_flash_attention_forward(q, k, v, return_lse=True, **kw)
        torch.cuda.synchronize()
        nfa.check_device_status(q.device)
        return o, lse, lib.bfa_launch_count() - n0
    finally:
        if prev is None:
            os.environ.pop("BFA_FWD_DECODE", None)
        else:
            os.environ["BFA_FWD_DECODE"] = prev


def _check(shape, dtype, mask_name, seed=0):
    b, hq, hkv, sq, sk, d = shape
    q, k, v, _ = _inputs(seed, b, hq, hkv, sq, sk, d, dtype)
    kw = dict(MASKS[mask_name])
    end_aligned = kw.pop("end_aligned", False)
    if kw.pop("alibi", False):
        kw["alibi_slope"] = torch.tensor([2.0 ** (-8.0 * (i + 1) / hq) for i in range(hq)])
    kw_dev = {**kw, **({"alibi_slope": kw["alibi_slope"].to(DEV)} if "alibi_slope" in kw else {})}
    ref_kw = dict(kw)
    if end_aligned:
        kw_dev["q_pos_offset"] = sk - sq
        ref_kw["q_offset"] = sk - sq
    qd, kd, vd = (t.to(DEV) for t in (q, k, v))
    o, lse, launches = _run(qd, kd, vd, kw_dev, decode=True)
    assert launches == 2, f"decode path not taken ({launches} launches)"
    o_ref, lse_ref = attention_forward(q, k, v, **ref_kw)
    tol = TOL[dtype]
    assert _err(o, o_ref) < tol, f"O err {_err(o, o_ref)}"
    assert _lse_err(lse, lse_ref) < LSE_RTOL, f"LSE err {_lse_err(lse, lse_ref)}"
    o2, lse2, _ = _run(qd, kd, vd, kw_dev, decode=False)
    assert _err(o, o2.cpu().double()) < tol
    assert _lse_err(lse, lse2.cpu().double()) < LSE_RTOL


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "b{}h{}k{}q{}s{}d{}".format(*s))
@pytest.mark.parametrize("mask_name", list(MASKS))
def test_decode_bf16(shape, mask_name):
    _check(shape, torch.bfloat16, mask_name)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32], ids=["f16", "f32"])
@pytest.mark.parametrize("shape", SHAPES[:3] + SHAPES[6:7], ids=lambda s: "b{}h{}k{}q{}s{}d{}".format(*s))
def test_decode_dtypes(shape, dtype):
    _check(shape, dtype, "none", seed=1)
    _check(shape, dtype, "causal_end", seed=2)


def test_decode_not_taken_for_many_rows():
    # G·Sq > 64 goes to the regular tcgen05 forward (one launch).
    q, k, v, _ = _inputs(5, 1, 8, 2, 20, 512, 128, torch.bfloat16)
    qd, kd, vd = (t.to(DEV) for t in (q, k, v))
    _, _, launches = _run(qd, kd, vd, {}, decode=True)
    assert launches == 1


def test_decode_scratch_comes_from_the_caller():
    """The partial O / LSE live in the caller's workspace: bfa_fwd_workspace_bytes
    sizes it, and without one bfa_fwd runs the regular forward (one launch)
    with the same result. The library keeps no memory pool of its own."""
    import ctypes
    lib = bfa_lib.load()
    q, k, v, _ = _inputs(9, 2, 8, 2, 1, 3000, 128, torch.bfloat16)
    qd, kd, vd = (t.to(DEV) for t in (q, k, v))
    pr = nfa._problem(qd, kd, False, 0, None, 128 ** -0.5, 0.0)
    need = lib.bfa_fwd_workspace_bytes(ctypes.byref(pr))
    assert need > 0 and need % 256 == 0
    o_ref, lse_ref, launches = _run(qd, kd, vd, {}, decode=True)
    assert launches == 2
    for ws_bytes in (0, need - 256):
        o = torch.empty_like(qd)
        lse = torch.empty(2, 8, 1, device=DEV)
        args = bfa_lib.FwdArgs()
        args.q, args.k, args.v, args.o = (bfa_lib.tensor(t) for t in (qd, kd, vd, o))
        args.lse = lse.data_ptr()
        ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=DEV)
        if ws_bytes:
            args.workspace, args.workspace_bytes = ws.data_ptr(), ws_bytes
        n0 = lib.bfa_launch_count()
        assert lib.bfa_fwd(ctypes.byref(pr), ctypes.byref(args),
                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
        torch.cuda.synchronize()
        assert lib.bfa_launch_count() - n0 == 1  # regular forward
        assert _err(o, o_ref.cpu().double()) < TOL[torch.bfloat16]
