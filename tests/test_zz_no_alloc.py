"""The allocation-free probability pass, redukt_b200_softmax_noalloc, through the C ABI.

Some callers cannot allocate device memory while they run: a host recording a CUDA graph (a
cudaMalloc cannot be captured), or one that decodes on a fixed device-memory budget behind a
caching allocator.  For them the library keeps the pass's scratch in a fixed array of its own.
This checks that entry point against the existing one, redukt_backend_forward_batch_probs, on two
calls in a row.  The file is named so pytest collects it last.
"""
import numpy as np
import pytest

from conftest import logsoftmax64
from redukt_b200.plugin import BackendResult, PluginBackend, PluginLibrary

pytestmark = pytest.mark.gpu

TOL_NATS = 1e-3  # the engine's parity tolerance on log-probabilities


def test_softmax_noalloc_matches_forward_batch_probs(ref_test_rbin):
    import torch

    b = PluginBackend(ref_test_rbin, library=PluginLibrary())
    try:
        V = b.vocab_size
        slots = [0, 1, 2]
        toks = [[5, 77, 1000], [42, 9, 311]]
        # logits of two consecutive steps, then the existing probability entry point on the same steps
        b.batch_init(len(slots))
        logits = [b.forward_batch(slots, t).copy() for t in toks]
        b.batch_init(len(slots))
        probs_ref = [b.forward_batch_probs(slots, t).copy() for t in toks]

        stream = torch.cuda.Stream()
        for step in range(2):  # two calls in a row share the library's scratch array
            d_logits = torch.from_numpy(logits[step]).cuda()
            d_probs = torch.full_like(d_logits, float("nan"))
            torch.cuda.synchronize()
            rc = b.libobj.softmax_noalloc(d_logits.data_ptr(), len(slots), V, d_probs.data_ptr(), stream.cuda_stream)
            assert rc == BackendResult.OK, b.libobj.last_error()
            stream.synchronize()
            got = d_probs.cpu().numpy()
            want = probs_ref[step]
            assert np.all(np.isfinite(got))
            lg = np.log(got.astype(np.float64))
            lw = np.log(want.astype(np.float64))
            assert np.max(np.abs(lg - lw)) <= TOL_NATS
            assert np.max(np.abs(lg - logsoftmax64(logits[step]))) <= TOL_NATS
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), "same kernels, same inputs"

        # sizes beyond the fixed scratch are refused with a clear error, nothing is launched
        big = torch.zeros((2, 70000), device="cuda")
        rc = b.libobj.softmax_noalloc(big.data_ptr(), 2, 70000, big.data_ptr(), 0)
        assert rc == BackendResult.INVALID_ARGUMENT
        assert "exceeds the fixed scratch" in b.libobj.last_error()
    finally:
        b.close()
