"""The C-ABI library loads and exports every entry point include/bfa.h declares.

CPU-only: the calls made here are rejected by argument validation before any
CUDA work, so no GPU is needed.
"""
import ctypes
import os
import re

import pytest

import bfa_lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "bfa.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|uint64_t|const char\*)\s+(bfa_\w+)\s*\(",
                                 text, re.M)))


def test_header_matches_binding_list():
    assert declared_symbols() == sorted(bfa_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = bfa_lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.bfa_abi_version() == bfa_lib.ABI_VERSION


def test_strerror_covers_every_status():
    lib = bfa_lib.load()
    for code in range(0, -7, -1):
        msg = lib.bfa_strerror(code).decode()
        assert msg and "unknown" not in msg
    assert "unknown" in lib.bfa_strerror(-99).decode()


def _problem(**kw):
    pr = bfa_lib.Problem()
    pr.batch, pr.heads_q, pr.heads_kv = 1, 4, 2
    pr.seqlen_q, pr.seqlen_k, pr.head_dim = 16, 16, 64
    pr.dtype, pr.scale = bfa_lib.DTYPE_BF16, 0.125
    for k, v in kw.items():
        setattr(pr, k, v)
    return pr


@pytest.mark.parametrize("kw,code", [
    ({"heads_q": 3, "heads_kv": 2}, -2),     # Hq % Hkv != 0 (reference asserts, :622)
    ({"head_dim": 300}, -3),                 # beyond 256
    ({"dtype": 7}, -3),                      # no such dtype
    ({"batch": -1}, -1),
    ({"sliding_window": -4}, -1),            # AttentionConfig rejects it too (:841-842)
    ({"soft_cap": -1.0}, -1),
    ({"heads_kv": 0}, -1),
])
def test_fwd_rejects_bad_problems_before_any_cuda_work(kw, code):
    lib = bfa_lib.load()
    args = bfa_lib.FwdArgs()
    assert lib.bfa_fwd(ctypes.byref(_problem(**kw)), ctypes.byref(args), None) == code


def test_null_arguments_are_rejected():
    lib = bfa_lib.load()
    assert lib.bfa_fwd(None, None, None) == -1
    assert lib.bfa_fwd(ctypes.byref(_problem()), ctypes.byref(bfa_lib.FwdArgs()), None) == -1
    ws = lib.bfa_bwd_workspace_bytes(ctypes.byref(_problem()))
    assert ws >= 4 * 16 * 4
    assert lib.bfa_bwd(ctypes.byref(_problem()), ctypes.byref(bfa_lib.BwdArgs()), None, 0, None) == -1


def test_fwd_accumulate_flag_is_checked():
    """bfa_fwd_args.accumulate is 0 or 1; any other value is rejected before
    any CUDA work (the pointers here are never dereferenced)."""
    lib = bfa_lib.load()
    args = bfa_lib.FwdArgs()
    for t in (args.q, args.k, args.v, args.o):
        t.data = 16
    args.lse = 16
    args.accumulate = 2
    assert lib.bfa_fwd(ctypes.byref(_problem()), ctypes.byref(args), None) == -1


def test_empty_problem_is_a_no_op():
    lib = bfa_lib.load()
    # B*Hq*Sq == 0: nothing to compute, nothing launched.
    assert lib.bfa_fwd(ctypes.byref(_problem(seqlen_q=0)), ctypes.byref(bfa_lib.FwdArgs()), None) == 0


def test_merge_partial_validates():
    lib = bfa_lib.load()
    t = bfa_lib.Tensor()
    assert lib.bfa_merge_partial(1, 1, 1, 0, t, 0, None, t, 0, None, None) == -1
    assert lib.bfa_merge_partial(1, 1, 1, 64, t, 9, None, t, 0, None, None) == -3
    assert lib.bfa_merge_partial(0, 1, 1, 64, t, 0, None, t, 0, None, None) == 0


def test_fwd_workspace_bytes_without_gpu():
    """bfa_fwd_workspace_bytes reports 0 for problems that never take the
    split-KV decoding path (and for invalid ones); the size of the decoding
    path's scratch is checked on the GPU (test_decode_gpu.py)."""
    lib = bfa_lib.load()
    assert lib.bfa_fwd_workspace_bytes(None) == 0
    assert lib.bfa_fwd_workspace_bytes(ctypes.byref(_problem(heads_q=3, heads_kv=2))) == 0
    # 4 q-heads per KV head x 256 rows: far above the 64 rows per KV head of the decoding path.
    assert lib.bfa_fwd_workspace_bytes(ctypes.byref(_problem(seqlen_q=256, seqlen_k=256))) == 0


def test_seqlen_q_bound():
    """Row pitches are padded to 64 in int32: lengths past INT32_MAX - 63 are
    rejected instead of overflowing."""
    lib = bfa_lib.load()
    pr = _problem(seqlen_q=2 ** 31 - 1)
    assert lib.bfa_fwd(ctypes.byref(pr), ctypes.byref(bfa_lib.FwdArgs()), None) == -1
    assert lib.bfa_bwd_workspace_bytes(ctypes.byref(pr)) == 0


def test_ctypes_structures_match_header_layout(tmp_path):
    """Size and every field offset of the ctypes mirrors equal the C
    structures of include/bfa.h, compiled here with gcc."""
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    structs = {"bfa_problem": bfa_lib.Problem, "bfa_tensor": bfa_lib.Tensor,
               "bfa_fwd_args": bfa_lib.FwdArgs, "bfa_bwd_args": bfa_lib.BwdArgs}
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "bfa.h"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in cls._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["  return 0;", "}"]
    src, exe = tmp_path / "layout.c", tmp_path / "layout"
    src.write_text("\n".join(lines) + "\n")
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {tuple(l.split()[:2]): int(l.split()[2]) for l in out if l.strip()}
    for cname, cls in structs.items():
        assert got[(cname, "size")] == ctypes.sizeof(cls), cname
        for field, _ in cls._fields_:
            assert got[(cname, field)] == getattr(cls, field).offset, (cname, field)


def test_last_error_is_a_string_before_any_failure():
    lib = bfa_lib.load()
    assert isinstance(lib.bfa_last_error(), bytes)
