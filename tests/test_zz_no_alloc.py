"""The allocation-free backward entry point (ffa_bwd_noalloc).

It serves callers that cannot allocate device memory — for example code that
is handed only its input and output buffers by a host framework, or that must
not call a device-synchronising cudaMalloc in the middle of a step.  It keeps
its scratch in an array compiled into the library.  This test calls it
directly through the C ABI, twice in a row (the second call sees the first
call's leftover scratch), and checks dq/dk/dv against the regular
workspace-taking ffa_bwd.  Both run the same deterministic kernels with a
fixed summation order, so the gradients must be bit-identical.
It lives in its own file collected last so a failure here never hides the
rest of the GPU suite.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _strides(t):
    from fastest_flash_attention_b200 import _lib
    return _lib.i64arr(t.stride(0), t.stride(1), t.stride(2))


def _call_noalloc(lib, do, q, k, v, o, lse, scale, causal, window, softcap):
    from fastest_flash_attention_b200 import _lib
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    B, Hq, Sq, D = q.shape
    st = lib.ffa_bwd_noalloc(
        do.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), _lib.DTYPE_CODE[q.dtype], B, Hq, k.shape[1], Sq, k.shape[2], D,
        _strides(q), _strides(k), _strides(v), _strides(o), _strides(do), _strides(dq), _strides(dk), _strides(dv),
        scale, int(causal), 0, int(window or 0), float(softcap or 0.0), _lib.err_word(q.device).data_ptr(),
        _lib.stream_of(q))
    _lib.check(st, "ffa_bwd_noalloc")
    return dq, dk, dv


def test_noalloc_backward_matches_workspace_backward_twice():
    from fastest_flash_attention_b200 import _lib
    from fastest_flash_attention_b200.attention import flash_bwd, flash_fwd
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(3)
    cases = [  # (B, Hq, Hkv, S, D, causal, window, softcap): different sizes so the scratch is reused dirty
        (2, 8, 2, 700, 128, True, None, None),
        (1, 4, 4, 333, 64, True, 100, 30.0),
    ]
    for B, Hq, Hkv, S, D, causal, window, softcap in cases:
        q = torch.randn(B, Hq, S, D, device="cuda", generator=g).to(torch.bfloat16)
        k = torch.randn(B, Hkv, S, D, device="cuda", generator=g).to(torch.bfloat16)
        v = torch.randn(B, Hkv, S, D, device="cuda", generator=g).to(torch.bfloat16)
        do = torch.randn(B, Hq, S, D, device="cuda", generator=g).to(torch.bfloat16)
        scale = 1 / math.sqrt(D)
        o, lse = flash_fwd(q, k, v, scale=scale, causal=causal, window=window, softcap=softcap)
        ref = flash_bwd(do, q, k, v, o, lse, scale=scale, causal=causal, window=window, softcap=softcap)
        got = _call_noalloc(lib, do, q, k, v, o, lse, scale, causal, window, softcap)
        torch.cuda.synchronize()
        _lib.check_device_errors(q.device)
        for a, b, nm in zip(got, ref, ("dq", "dk", "dv")):
            assert torch.equal(a, b), f"{nm}: differs from ffa_bwd (max abs {(a.float() - b.float()).abs().max().item():.3e})"


def test_noalloc_rejects_oversized_problem():
    from fastest_flash_attention_b200 import _lib
    lib = _lib.load()
    s = _lib.i64arr(0, 0, 0)
    # 9 heads x 128 x 1024 rows > 2^20: rejected before any pointer is used
    st = lib.ffa_bwd_noalloc(1, 1, 1, 1, 1, 1, 16, 16, 16, 1, 1, 9, 9, 128 * 1024, 16, 128, s, s, s, s, s, s, s, s,
                             1.0, 1, 0, 0, 0.0, None, None)
    assert st == _lib.FFA_ERR_UNSUPPORTED
    assert b"FFA_BWD_NOALLOC_MAX_ROWS" in lib.ffa_last_error()
