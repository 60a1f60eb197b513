"""Bounded device waits that run out end the step with an error, and the device stays usable.

Every wait in the engine's kernels (the fused step's grid barriers and copy waits, the
tensor-core pipelines' mbarrier waits) gives up after a time limit, sets a bit of the device error
word and lets the kernel return; the host turns the word into FORWARD_FAILED.  These tests make one
wait run out on purpose with the engine's test settings: the limit is shortened to 2 ms and one
arrival (fused step) or one copy (tensor-core tile) is withheld, so the waiting side sees a flag that
nothing sets.  Nothing faults: the waits simply give up.  The next normal step must then return the
same bits as a step that never saw the failure.
"""
import numpy as np
import pytest

from conftest import q8, shared_backend
from redukt_b200.plugin import BackendResult, PluginError
from redukt_b200.workload import zipf_tokens

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("kind,n,fused,word", [(1, 8, 1, 0x4), (2, 40, 0, 0x2)])
def test_wait_runs_out_then_next_step_is_correct(small_gauss_rbin, kind, n, fused, word):
    b = shared_backend(q8(small_gauss_rbin))
    V = b.vocab_size
    toks = zipf_tokens(n, 3, vocab=V, seed_base=901)
    slots = list(range(n))
    try:
        b.set_option("fused", fused)
        b.set_option("graphs", 0)
        # reference: the same two steps with nothing withheld
        b.batch_init(n)
        want = [b.forward_batch(slots, toks[:, t]).copy() for t in range(2)]
        b.batch_init(n)
        b.set_option("wait_limit_us", 2000)
        b.set_option("wait_test", kind)
        with pytest.raises(PluginError) as ei:
            b.forward_batch(slots, toks[:, 0])
        assert ei.value.code == BackendResult.FORWARD_FAILED
        assert f"device error word 0x{word:x}" in str(ei.value), str(ei.value)
        b.set_option("wait_limit_us", 0)
        # the failed step may have written part of the state: start the streams again
        b.batch_reset()
        got = [b.forward_batch(slots, toks[:, t]).copy() for t in range(2)]
        for t in range(2):
            assert np.array_equal(bits(got[t]), bits(want[t])), t
        assert b.device_error() == 0
    finally:
        b.set_option("wait_test", 0)
        b.set_option("wait_limit_us", 0)
        b.set_option("graphs", 1)
        b.set_option("fused", 1)
