"""The fused small-batch step (one persistent kernel per step for up to 32 streams) against the
per-kernel step: logits and both state tensors must agree bit for bit, for every batch size the
fused kernel covers, with slot resets and the device-side periodic reset.

The per-kernel path is itself checked against the CPU oracle and against the reference's own
golden vectors (test_gpu_parity.py), and the fused path runs all of those tests too (it is the
default for Q8 batches of up to 32 streams)."""
import math

import numpy as np
import pytest

from conftest import q8, shared_backend
from redukt_b200.workload import zipf_tokens

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def run(b, fused, n, toks, slots, cap, resets):
    b.set_option("fused", fused)
    b.batch_init(cap)
    out = []
    for t in range(toks.shape[1]):
        if t in resets:
            b.batch_reset([slots[s] for s in resets[t]])
        out.append(b.forward_batch(slots, toks[:, t]).copy())
    states = [b.get_state(slots[s]) for s in (0, n - 1)]
    return np.stack(out, 1), states


@pytest.mark.parametrize("fused", [1])
@pytest.mark.parametrize("quant", ["q8", "q8row"])
@pytest.mark.parametrize("model", ["reftest", "gauss_small", "mamba130m"])
def test_fused_step_bit_identical_to_kernel_path(ref_test_rbin, small_gauss_rbin, mamba130m_rbin, model, quant,
                                                 fused):
    base = {"reftest": ref_test_rbin, "gauss_small": small_gauss_rbin, "mamba130m": mamba130m_rbin}[model]
    b = shared_backend(q8(base, quant == "q8row"))
    V = b.vocab_size
    sizes = (1, 3, 8, 9, 17, 32) if model != "mamba130m" else (1, 5, 32)
    try:
        for n in sizes:
            steps = 4
            toks = zipf_tokens(n, steps, vocab=V, seed_base=31 * n)
            cap = n + 5
            mult = next(m for m in range(3, cap + 3) if math.gcd(m, cap) == 1)  # a permutation of the slots
            slots = [(mult * s + 2) % cap for s in range(n)]
            resets = {2: [s for s in range(n) if s % 4 == 1]}
            got, st_f = run(b, fused, n, toks, slots, cap, resets)
            want, st_k = run(b, 0, n, toks, slots, cap, resets)
            assert np.array_equal(bits(got), bits(want)), (model, quant, n, fused)
            for (cf, sf), (ck, sk) in zip(st_f, st_k):
                assert np.array_equal(bits(cf), bits(ck)) and np.array_equal(bits(sf), bits(sk)), (model, quant, n, fused)
            assert b.device_error() == 0
    finally:
        b.set_option("fused", 1)


def test_fused_step_device_periodic_reset(small_gauss_rbin):
    b = shared_backend(q8(small_gauss_rbin))
    V = b.vocab_size
    n, steps = 6, 9
    toks = zipf_tokens(n, steps, vocab=V, seed_base=5)
    outs = {}
    try:
        for fused in (1, 0):
            b.set_option("fused", fused)
            b.batch_init(8)
            b.set_reset_every(4)
            outs[fused] = np.stack([b.forward_batch(list(range(n)), toks[:, t]).copy() for t in range(steps)], 1)
            b.set_reset_every(0)
    finally:
        b.set_option("fused", 1)
        b.set_reset_every(0)
    assert np.array_equal(bits(outs[1]), bits(outs[0]))


def test_fused_step_probs_and_device_path(small_gauss_rbin):
    torch = pytest.importorskip("torch")
    b = shared_backend(q8(small_gauss_rbin))
    V = b.vocab_size
    n = 7
    toks = zipf_tokens(n, 3, vocab=V, seed_base=11)
    outs = {}
    try:
        for fused in (1, 0):
            b.set_option("fused", fused)
            b.batch_init(n)
            p = [b.forward_batch_probs(list(range(n)), toks[:, t]).copy() for t in range(2)]
            dev = torch.device("cuda:0")
            d_slots = torch.arange(n, dtype=torch.int32, device=dev)
            d_tok = torch.from_numpy(toks[:, 2].astype(np.int32)).to(dev)
            d_out = torch.empty((n, V), dtype=torch.float32, device=dev)
            b.forward_batch_device(n, d_slots.data_ptr(), d_tok.data_ptr(), d_out.data_ptr())
            torch.cuda.synchronize()
            outs[fused] = (np.stack(p), d_out.cpu().numpy())
    finally:
        b.set_option("fused", 1)
    assert np.array_equal(bits(outs[1][0]), bits(outs[0][0]))
    assert np.array_equal(bits(outs[1][1]), bits(outs[0][1]))
