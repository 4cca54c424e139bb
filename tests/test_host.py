"""CPU-side checks: the C-ABI library loads and exports every symbol the
header declares, host-side API behaviour (config, block-size heuristic,
block masks, shape errors, no CPU fallback).  No kernel is launched."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (ROOT / "include" / "ffa_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ffa_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from fastest_flash_attention_b200 import _lib
    lib = _lib.load()
    names = declared_symbols()
    assert "ffa_fwd" in names
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ffa_b200.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_library_version_and_error_string():
    from fastest_flash_attention_b200 import _lib
    lib = _lib.load()
    assert lib.ffa_version() == 10000
    assert isinstance(lib.ffa_last_error(), bytes)


def test_invalid_arguments_rejected_without_launch():
    """Null pointers / bad head counts return FFA_ERR_INVALID_ARG before any CUDA call."""
    from fastest_flash_attention_b200 import _lib
    lib = _lib.load()
    s = _lib.i64arr(0, 0, 0)
    st = lib.ffa_fwd(None, None, None, None, None, 1, 1, 1, 1, 1, 1, 128, 128, s, s, s, s, 1.0, 0, 0, 0, 0.0,
                     None, 0, 0, 0, 0, None, None)
    assert st == _lib.FFA_ERR_INVALID_ARG
    st = lib.ffa_fwd(1, 1, 1, 16, None, 1, 1, 3, 2, 1, 1, 128, 128, s, s, s, s, 1.0, 0, 0, 0, 0.0,
                     None, 0, 0, 0, 0, None, None)
    assert st == _lib.FFA_ERR_INVALID_ARG
    st = lib.ffa_fwd(1, 1, 1, 16, None, 1, 1, 1, 1, 1, 1, 96, 96, s, s, s, s, 1.0, 0, 0, 0, 0.0,
                     None, 0, 0, 0, 0, None, None)
    assert st == _lib.FFA_ERR_UNSUPPORTED


def test_cpu_tensors_raise_no_fallback():
    import fastest_flash_attention_b200 as ffa
    q = torch.randn(1, 2, 8, 64)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ffa.fastest_flash_attn_forward(q, q, q)


def test_auto_block_size_matches_reference_rules():
    from fastest_flash_attention_b200 import auto_select_block_size
    for S in (1, 7, 64, 100, 1000, 8192):
        for D in (16, 64, 128, 192):
            bs = auto_select_block_size(S, S, D)
            assert bs & (bs - 1) == 0 and 16 <= bs <= 256
    assert auto_select_block_size(4096, 4096, 16) == 256
    assert auto_select_block_size(4096, 4096, 128) == 32


def test_config_defaults_match_reference():
    from fastest_flash_attention_b200 import AttentionConfig
    c = AttentionConfig()
    assert (c.block_size_q, c.block_size_kv, c.causal, c.page_size, c.pipeline_stages) == (0, 0, False, 64, 2)
    assert c.resolve_block_sizes(1024, 1024, 64) == (64, 64)


def test_kernel_dtype_selection():
    """fp32 (and fp64) inputs compute in fp32 unless compute_dtype asks for a
    16-bit type; 16-bit inputs keep their type (cpu_reference.py:28-32)."""
    from fastest_flash_attention_b200.attention import kernel_dtype, _ATTN_DTYPE_CODE
    f32, f64 = torch.zeros(1, dtype=torch.float32), torch.zeros(1, dtype=torch.float64)
    assert kernel_dtype(f32) == torch.float32
    assert kernel_dtype(f64) == torch.float32
    assert kernel_dtype(f32, torch.float16) == torch.float16
    assert kernel_dtype(f32, torch.bfloat16) == torch.bfloat16
    assert kernel_dtype(torch.zeros(1, dtype=torch.bfloat16), torch.float16) == torch.bfloat16
    assert _ATTN_DTYPE_CODE == {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def test_fp32_entry_points_reject_misaligned_strides_without_launch():
    """ffa_fwd with FFA_DTYPE_F32 validates 16-byte alignment and strides that
    are multiples of 4 elements before touching the GPU."""
    from fastest_flash_attention_b200 import _lib
    lib = _lib.load()
    s = _lib.i64arr(64 * 65, 64 * 65, 65)  # seq stride 65: not a multiple of 4 floats
    st = lib.ffa_fwd(16, 16, 16, 16, None, 2, 1, 1, 1, 64, 64, 64, 64, s, s, s, s, 0.125, 0, 0, 0, 0.0,
                     None, 0, 0, 64, 64, None, None)
    assert st == 1  # FFA_ERR_INVALID_ARG
