"""Device-side waits give up instead of hanging: the diagnostic kernel
waits, bounded, on a barrier that nothing completes; the give-up is
counted where the host can read it and the context stays usable."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports(ctx, hp):
    hp.wait_timeouts(reset=True)
    hp.check_bounded_wait(1000)
    hp.check_bounded_wait(1000)
    assert hp.wait_timeouts(reset=True) == 2
    assert hp.wait_timeouts() == 0
    # the context still works afterwards
    x = np.arange(1000, dtype=np.int32)
    dx = ctx.allocate("i32", x.size)
    dx.copy_from(x)
    assert hp.reduce_sum_i32(dx) == orc.sum_i32(x)
