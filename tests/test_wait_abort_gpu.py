"""The bounded pipeline waits of the tcgen05 prefix pass, made to run out on purpose.

Every mbarrier wait of the prefix kernel gives up after a fixed number of
polls; the kernel then sets its abort flag, drains the copies and MMAs it has
issued, frees its tensor memory and ends, and qa_check_device_error reports
it. With the test hook qa_set_pipeline_wait_limit(1) a wait that is not
already complete gives up at once, so the abort path runs without any fault:
the launch must end, the flag must be reported, and the next launch (default
limit) must be correct in the same context.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qattention_b200 import _lib
    from qattention_b200 import ragged_attn as ra


def _inputs():
    g = torch.Generator().manual_seed(41)
    B, L, N, Hq, Hkv, D = 2, 4096, 64, 8, 2, 128
    Q = torch.randn(B, N, Hq, D, generator=g).half()
    K = torch.randn(B, L, Hkv, D, generator=g).half()
    V = torch.randn(B, L, Hkv, D, generator=g).half()
    return Q, K, V


def test_prefix_waits_run_out_and_report():
    Q, K, V = _inputs()
    Qd, Kd, Vd = Q.cuda(), K.cuda(), V.cuda()
    assert _lib.device_error() == 0
    L = _lib.lib()
    try:
        assert L.qa_set_pipeline_wait_limit(1) == 0
        ra.prefix_attention_with_lse(Qd, Kd, Vd)
        torch.cuda.synchronize()  # the launch ended (no hang, no fault)
        flag = _lib.device_error()
    finally:
        L.qa_set_pipeline_wait_limit(0)
    assert flag & 1, "the prefix kernel did not report its timed-out waits"
    # the context is usable and the default limit gives the right result
    O, LSE = ra.prefix_attention_with_lse(Qd, Kd, Vd)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    B, N, Hq, D = Q.shape
    r = Hq // K.shape[2]
    for s in range(B):  # dense attention over every prefix key (fp32), GQA by repeating KV heads
        q = Q[s].float().permute(1, 0, 2)                              # [Hq, N, D]
        k = K[s].float().repeat_interleave(r, 1).permute(1, 0, 2)      # [Hq, L, D]
        v = V[s].float().repeat_interleave(r, 1).permute(1, 0, 2)
        ref = torch.softmax(q @ k.transpose(1, 2) / D ** 0.5, -1) @ v  # [Hq, N, D]
        assert torch.allclose(O[s].float().cpu(), ref.permute(1, 0, 2), atol=1e-2, rtol=1e-2)
