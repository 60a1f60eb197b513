"""A bad entry on the device-resident step path rejects only its own stream.

redukt_b200_forward_batch_device checks slots and tokens on the device.  The host-buffer calls
return INVALID_ARGUMENT "before any launch, with no state change" (docs/api/PLUGIN-FFI-V2.md:74);
the device path cannot return early, so a bad entry must instead leave its slot's state exactly as
it was, write an all-zero output row, set bit 0 of the device error word, and change nothing for the
other streams of the batch.  Checked for the fused Q8 step (n <= 32), the per-kernel Q8 step
(n > 32), the F32 step and the RWKV-7 step.
"""
import os

import numpy as np
import pytest

from conftest import q8, shared_backend
from redukt_b200 import rwkv7_rbin as R
from redukt_b200.workload import zipf_tokens

pytestmark = pytest.mark.gpu

BAD_POS = 3


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def state_of(b, slot):
    return b.rwkv_state(slot) if b.is_rwkv else b.get_state(slot)


def check_reject(b, n, toks):
    """Slots 0..n-1 (device path, one bad token) and 64..64+n-1 (host path, the good streams only)
    start from the same history; one step later every good row agrees bit for bit."""
    import torch

    V = b.vocab_size
    warm = toks.shape[1] - 1
    a_slots = list(range(n))
    h_slots = [64 + s for s in range(n)]
    b.batch_init(64 + n)
    for t in range(warm):  # identical histories in both slot sets
        b.forward_batch(a_slots, toks[:, t])
        b.forward_batch(h_slots, toks[:, t])
    assert b.device_error() == 0
    before = state_of(b, a_slots[BAD_POS])
    step = toks[:, warm].astype(np.int64).copy()
    step[BAD_POS] = V  # token >= vocab
    dev = torch.device("cuda:0")
    d_slots = torch.tensor(a_slots, dtype=torch.int32, device=dev)
    d_tok = torch.from_numpy(step.astype(np.int32)).to(dev)
    d_out = torch.full((n, V), float("nan"), dtype=torch.float32, device=dev)
    b.forward_batch_device(n, d_slots.data_ptr(), d_tok.data_ptr(), d_out.data_ptr())
    torch.cuda.synchronize()
    got = d_out.cpu().numpy()
    assert b.device_error() & 1, "a bad token sets bit 0 of the device error word"
    assert b.device_error() == 0, "reading the word clears it"
    after = state_of(b, a_slots[BAD_POS])
    for x, y in zip(before, after):
        assert np.array_equal(bits(x), bits(y)), "the rejected stream's slot state changed"
    assert np.array_equal(bits(got[BAD_POS]), np.zeros(V, np.uint32)), "a rejected row is all +0.0"
    good = [s for s in range(n) if s != BAD_POS]
    want = b.forward_batch([h_slots[s] for s in good], toks[good, warm])
    assert np.array_equal(bits(got[good]), bits(want))
    # the rejected slot still steps normally afterwards, from its unchanged state: it matches its
    # twin in the host slot set once that twin has been given the same token
    nxt = toks[:, warm]
    b.forward_batch([h_slots[BAD_POS]], [int(nxt[BAD_POS])])  # the twin (was left out above)
    r1 = b.forward_batch([a_slots[BAD_POS]], [int(nxt[BAD_POS])])
    assert b.device_error() == 0
    twin_state = state_of(b, h_slots[BAD_POS])
    for x, y in zip(state_of(b, a_slots[BAD_POS]), twin_state):
        assert np.array_equal(bits(x), bits(y))
    assert np.all(np.isfinite(r1))


@pytest.mark.parametrize("case", ["q8_fused", "q8_kernels", "f32"])
def test_bad_token_rejects_only_its_stream_mamba(small_gauss_rbin, case):
    path = small_gauss_rbin if case == "f32" else q8(small_gauss_rbin)
    b = shared_backend(path)
    n = 8 if case != "q8_kernels" else 40  # above 32 streams the per-kernel step runs
    toks = zipf_tokens(n, 4, vocab=b.vocab_size, seed_base=77)
    check_reject(b, n, toks)


def test_bad_token_rejects_only_its_stream_rwkv7(model_dir):
    path = R.ensure_model(os.path.join(model_dir, "rwkv7_small.rbin"), R.RWKV7_TEST_DIMS)
    b = shared_backend(path)
    n = 8
    toks = R.byte_tokens(n, 3, seed=19)
    check_reject(b, n, toks)
