"""The dQ kernels' fused Δ prologue (head dims 64, 128, 256): a backward call with
both the Δ and dQ phases has the dQ kernel form Δ = rowsum(O∘dO) and the
row statistic lse2 itself, and write them for the dK/dV kernel that runs
after it. Here the workspace rows it writes are compared with the separate Δ
pass's (a call with the Δ phase alone), including padded rows and query
tiles that see no key, and the gradients of one fused call with those of
separate phase calls."""
import pytest
import torch

import bfa_lib
import npu_flash_attention as nfa
from test_parity_gpu import DEV, _inputs

pytestmark = pytest.mark.gpu


def _rowstats(ws, b, hq, sq):
    pad = (sq + 63) // 64 * 64
    n = b * hq * pad
    stride = (n * 4 + 255) // 256 * 256
    delta = ws[:n * 4].view(torch.float32).view(b, hq, pad)
    lse2 = ws[stride:stride + n * 4].view(torch.float32).view(b, hq, pad)
    return delta.clone(), lse2.clone()


CASES = [
    # (dtype, d, hq, hkv, sq, sk, options)
    (torch.bfloat16, 128, 4, 2, 520, 520, dict(causal=True)),
    (torch.float16, 64, 4, 1, 300, 300, dict()),
    (torch.bfloat16, 128, 2, 2, 640, 256, dict(causal=True, alibi=True)),
    (torch.bfloat16, 128, 2, 1, 384, 200, dict(causal=True, k_pos_offset=200)),  # rows 0..199 see no key
    (torch.bfloat16, 64, 2, 2, 129, 129, dict(causal=True, soft_cap=20.0, sliding_window=50)),
    (torch.bfloat16, 256, 4, 2, 520, 520, dict(causal=True, soft_cap=30.0)),
    (torch.float16, 256, 2, 1, 300, 200, dict(causal=True, k_pos_offset=100)),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "{}-d{}-sq{}-sk{}-{}".format(
    str(c[0]).split(".")[-1], c[1], c[4], c[5], "-".join(sorted(c[6])) or "full"))
def test_fused_delta_matches_delta_pass(case):
    dt, d, hq, hkv, sq, sk, opts = case
    opts = dict(opts)
    if opts.pop("alibi", False):
        opts["alibi_slope"] = torch.tensor([2.0 ** (-8.0 * (i + 1) / hq) for i in range(hq)], device=DEV)
    q, k, v, go = (t.to(DEV) for t in _inputs(sq + sk + d, 2, hq, hkv, sq, sk, d, dt))
    o, lse = nfa.npu_flash_attention_forward(q, k, v, return_lse=True, **opts)
    lib = bfa_lib.load()
    pr = nfa._problem(q, k, opts.get("causal", False), opts.get("sliding_window", 0), None,
                      1.0, opts.get("soft_cap", 0.0))
    nbytes = lib.bfa_bwd_workspace_bytes(pr)
    ws_a = torch.full((nbytes,), 0xAB, dtype=torch.uint8, device=DEV)
    ws_b = torch.full((nbytes,), 0xCD, dtype=torch.uint8, device=DEV)
    # Separate passes: Δ alone, then dK/dV, then dQ.
    sep = tuple(torch.empty_like(t) for t in (q, k, v))
    for ph in (bfa_lib.PHASE_DELTA, bfa_lib.PHASE_DKDV, bfa_lib.PHASE_DQ):
        nfa.npu_flash_attention_backward(q, k, v, o, lse, go, _phases=ph, _workspace=ws_a,
                                         _outputs=(sep[0], sep[1], sep[2]), **opts)
    # One call: the dQ kernel forms Δ, then dK/dV.
    fused = nfa.npu_flash_attention_backward(q, k, v, o, lse, go, _workspace=ws_b, **opts)
    torch.cuda.synchronize()
    nfa.check_device_status(DEV)
    d_a, l_a = _rowstats(ws_a, 2, hq, sq)
    d_b, l_b = _rowstats(ws_b, 2, hq, sq)
    assert torch.equal(l_a, l_b), "lse2 rows differ"
    assert torch.allclose(d_a, d_b, rtol=1e-5, atol=1e-5), (d_a - d_b).abs().max().item()
    assert (d_b[:, :, sq:] == 0).all() and torch.isinf(l_b[:, :, sq:]).all()
    for a, b in zip(sep, fused):
        assert torch.allclose(a.float(), b.float(), rtol=2e-2, atol=2e-2)
