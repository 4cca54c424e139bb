"""Bounded in-kernel waits: with a wait limit far shorter than a tile copy,
the forward's waits expire, the kernel records its site code in the error
word, lets its copies and MMAs in flight finish (draining waits keep a
multi-second floor whatever the limit) and returns.  The host sees
FFA_ERR_DEVICE_TIMEOUT and the CUDA context stays usable: the next call with
the default limit is correct.  No fault, trap or hang is involved."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_and_context_survives():
    import fastest_flash_attention_b200 as ffa
    from fastest_flash_attention_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device="cuda").manual_seed(9)
    q, k, v = (torch.randn(1, 2, 1024, 128, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
    _lib.check_device_errors(dev)
    lib.ffa_set_wait_limit_ns(1)  # 1 ns: every wait that is not already complete expires
    try:
        with pytest.raises(RuntimeError, match="FFA_ERR_DEVICE_TIMEOUT") as e:
            # the call raises itself when FFA_SYNC_CHECK is on; else the check does
            ffa.fastest_flash_attn_forward(q, k, v, causal=True)
            torch.cuda.synchronize()
            _lib.check_device_errors(dev)
        code = int(str(e.value).split("site 0x")[1].split()[0], 16)
        assert 0x100 <= code < 0x200, hex(code)  # a forward site
    finally:
        lib.ffa_set_wait_limit_ns(0)  # back to the default
    o = ffa.fastest_flash_attn_forward(q, k, v, causal=True)[0]
    torch.cuda.synchronize()
    _lib.check_device_errors(dev)
    s = (q[0].float() @ k[0].float().transpose(-1, -2)) / math.sqrt(128)
    s = s.masked_fill(torch.ones(1024, 1024, device=dev, dtype=torch.bool).triu(1), float("-inf"))
    ref = torch.softmax(s, -1) @ v[0].float()
    assert (o[0].float() - ref).abs().max().item() <= 2e-2
