"""A bounded device-side wait that runs out reaches the caller.

The tensor-core kernels bound every mbarrier wait; when one expires the
kernel records a code in its status word and skips its output.  The library
reads that word whenever it synchronises (tp_synchronize, tp_comm_sync) and
returns TP_ERR_TIMEOUT, so a lost wait is an error, not silently wrong
numbers.  tp_wait_probe makes that happen without any copy or tensor memory:
one CTA waits, through the kernels' own wait function, on an mbarrier that
nothing arrives on, with a 2 ms limit.
"""
import pytest

from tpcuda._lib import TpError, check

pytestmark = pytest.mark.gpu

TP_ERR_TIMEOUT = -5


def test_expired_wait_is_reported_by_synchronize_once(cuda_rt):
    rt = cuda_rt
    rt.synchronize()  # nothing pending
    check(rt.lib.tp_wait_probe(2_000_000))
    with pytest.raises(TpError) as e:
        rt.synchronize()
    assert e.value.status == TP_ERR_TIMEOUT
    assert "code 99" in str(e.value)
    rt.synchronize()  # the word was cleared when it was reported
    # the context stays usable
    h = rt.full([3], 2.5, "float32")
    assert rt.toList(h["id"]) == [2.5, 2.5, 2.5]
    rt.destroy(h["id"])


def test_probe_limit_is_checked(cuda_rt):
    assert cuda_rt.lib.tp_wait_probe(10) != 0
    assert cuda_rt.lib.tp_wait_probe(3_000_000_000) != 0
