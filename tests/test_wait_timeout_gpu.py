"""The kernels' bounded waits, made to run out on purpose (no GPU fault, no hang).

cfk_test_wait_timeout launches one warp that waits on a barrier no thread ever arrives on,
through the same waiting loop every kernel uses.  The wait gives up after its limit (a few
milliseconds here), records 1 (a barrier wait ran past its limit) in the device status word and
the kernel returns normally.  The tests check that word, that clearing it works, that the
per-device limit (cfk_set_wait_limit_ns) is what the loop obeys, that torch_ops' status check
raises, and that a real launch afterwards runs clean and correct.
"""

import math

import pytest
import torch

import oracle
from conftest import assert_close_bf16

pytestmark = pytest.mark.gpu

TIMEOUT_BARRIER = 1  # kStatusTimeoutBarrier


def _selftest(limit_ns):
    from colabfold_legacy_kernels import cabi
    result = torch.zeros(1, dtype=torch.int32, device="cuda")
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream()
    a.record(stream)
    cabi.call("cfk_test_wait_timeout", stream.cuda_stream, int(limit_ns), result.data_ptr())
    b.record(stream)
    torch.cuda.synchronize()
    return int(result.item()), a.elapsed_time(b)


def test_wait_gives_up_and_records_status(cuda_device):
    from colabfold_legacy_kernels import cabi
    cabi.clear_device_status()
    assert cabi.device_status() == 0
    result, ms = _selftest(5_000_000)  # 5 ms
    assert result == 1, "the wait on a barrier nobody arrives on did not give up"
    assert 4.0 <= ms < 500.0, ms
    assert cabi.device_status() == TIMEOUT_BARRIER
    cabi.clear_device_status()
    assert cabi.device_status() == 0


def test_device_wait_limit_is_what_the_loop_obeys(cuda_device):
    from colabfold_legacy_kernels import cabi
    old = cabi.get_wait_limit_ns()
    assert old == 1_000_000_000
    try:
        cabi.set_wait_limit_ns(3_000_000)  # 3 ms
        assert cabi.get_wait_limit_ns() == 3_000_000
        cabi.clear_device_status()
        result, ms = _selftest(0)  # 0: the device's limit
        assert result == 1
        assert 2.5 <= ms < 500.0, ms
        assert cabi.device_status() == TIMEOUT_BARRIER
    finally:
        cabi.set_wait_limit_ns(old)
        cabi.clear_device_status()
    assert cabi.get_wait_limit_ns() == old
    with pytest.raises(cabi.CfkError) as e:
        cabi.set_wait_limit_ns(10)
    assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT


def test_status_check_raises_then_real_launch_runs_clean(cuda_device):
    from colabfold_legacy_kernels import cabi, torch_ops
    cabi.clear_device_status()
    _selftest(1_000_000)
    with pytest.raises(cabi.CfkError) as e:
        torch_ops.check_status(cuda_device)
    assert "gave up" in e.value.message
    cabi.clear_device_status()
    torch_ops.check_status(cuda_device)  # clean again
    # the context is usable: a real attention forward + backward, checked against the oracle
    g = torch.Generator().manual_seed(5)
    n, h, s, d = 3, 2, 200, 32
    q, k, v, dout = (torch.randn(n, h, s, d, generator=g).to(torch.bfloat16) for _ in range(4))
    bias = torch.randn(h, s, s, generator=g).to(torch.bfloat16)
    kmask = (torch.rand(n, s, generator=g) > 0.1).to(torch.uint8)
    scale = 1 / math.sqrt(d)
    t = [x.cuda() for x in (q, k, v, bias, kmask, dout)]
    out, lse = torch_ops.attention_fwd(*t[:5], scale)
    dq, dk, dv, dbias = torch_ops.attention_bwd(*t[:5], out, lse, t[5], scale)
    torch_ops.check_status(cuda_device)
    ref_out, _ = oracle.attention_fwd(q, k, v, bias, kmask, scale)
    assert_close_bf16(out, ref_out, "out after a timed-out self-test")
    r = oracle.attention_bwd(q, k, v, bias, kmask, out.cpu(), lse.cpu(), dout, scale)
    assert_close_bf16(dq, r[0], "dq after a timed-out self-test")
    assert cabi.device_status() == 0
