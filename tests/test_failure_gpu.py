"""The device-side failure path, exercised without faulting or hanging a GPU.

Every pipelined kernel waits on mbarriers through one bounded wait; when a
wait gives up it records a code in a status word, drains what it has in
flight and returns.  gpa_wait_selftest runs that wait on a barrier nothing
arrives on, with a 1 ms limit: the host must see KernelTimeout, and the same
context must then run a normal attention launch correctly.  The persistent
per-device status word that production launches share raises once at the
forward's check and is then clear.
"""
import pytest
import torch

from oracle import gpa_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from gpa_vggt_b200 import build, _lib
    build.build()
    _lib.load()


def test_wait_that_nothing_satisfies_times_out_and_context_survives():
    from gpa_vggt_b200 import kernels
    with pytest.raises(kernels.KernelTimeout):
        kernels.wait_selftest(1_000_000)           # 1 ms
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 2, 300, 64, generator=g).bfloat16() for _ in range(3))
    o = kernels.attention(q.cuda(), k.cuda(), v.cuda(), None, 0.125)
    ref = O.attention_keybias(q, k, v, None, 0.125)
    err = float((o.cpu().double() - ref).norm() / ref.norm())
    assert err < 1e-2


def test_persistent_status_word_raises_once():
    from gpa_vggt_b200 import kernels
    w = kernels.device_status_word("cuda")
    kernels.check_device_status("cuda")            # clear
    w.fill_(1)                                     # as a kernel whose wait gave up would
    with pytest.raises(kernels.KernelTimeout):
        kernels.check_device_status("cuda")
    kernels.check_device_status("cuda")            # cleared by the raise


def test_selftest_rejects_limits_outside_its_range():
    from gpa_vggt_b200 import _lib, kernels
    with pytest.raises(_lib.GpaError):
        kernels.wait_selftest(10)
