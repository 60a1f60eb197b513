"""The coder CDF on the device (redukt_b200_cdf_device / redukt_b200_cdf) against the C oracle.

The reference turns each row of (ensemble) logits into the range coder's 24-bit frequency table
on the host: cdf_from_logits_with under numeric contract fmath-v1 (src/application/codec.rs:785-798)
then Cdf::from_probs (src/domain/coder.rs:43-82).  The result is integer data that the encoder and
the decoder must agree on bit for bit, so every comparison here is exact.

CPU tests pin the oracle: its exp against the reference's golden bit patterns
(src/domain/fmath.rs:525-550, extracted by golden/make_exp_golden.py), its CDF against a
pure-Python restatement on small rows, and the exactness argument of the device kernel's
binade-blocked summation against plain sequential summation.  GPU tests compare the kernel with the
oracle on ragged, masked, peaked, flat and full-size rows (rows of up to 53,248 logits keep their
workspace in shared memory, longer ones in the output row: both sides of that limit are covered),
and the encoder / decoder queries.
"""
import json
import math
import os
import struct
import sys

import numpy as np
import pytest

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
TOTAL = 1 << 24


def _bits(x: float) -> int:
    return struct.unpack("<Q", struct.pack("<d", x))[0]


def _dbl(u: int) -> float:
    return struct.unpack("<d", struct.pack("<Q", u))[0]


# ----------------------------------------------------------------------------------------------
# CPU: the oracle
# ----------------------------------------------------------------------------------------------

def test_oracle_exp_matches_reference_golden_bits():
    g = json.load(open(os.path.join(HERE, "golden", "exp_f64_golden.json")))
    assert len(g["pairs"]) == 24
    for x, want in g["pairs"]:
        got = _bits(O.exp_f64(_dbl(int(x, 16))))
        assert got == int(want, 16), f"exp({_dbl(int(x, 16))!r})"


def test_oracle_exp_within_one_ulp_of_libm():
    rng = np.random.default_rng(7)
    xs = np.concatenate([-60.0 * rng.random(20000), -745.0 + 1454.0 * rng.random(20000)])
    worst = 0
    for x in xs:
        a, b = _bits(O.exp_f64(float(x))), _bits(math.exp(float(x)))
        worst = max(worst, abs(a - b))
    assert worst <= 1


def test_exp_table_header_is_current():
    sys.path.insert(0, os.path.join(ROOT, "redukt_b200", "csrc"))
    try:
        import gen_exp_table
    finally:
        sys.path.pop(0)
    text = open(os.path.join(ROOT, "redukt_b200", "csrc", "rk_exp_table.h")).read()
    words = [int(w, 16) for w in __import__("re").findall(r"0x([0-9a-f]{16})ull", text)]
    assert words == gen_exp_table.table()
    assert words[:4] == [0, 0x3ff0000000000000, 0x3c9b3b4f1a88bf6e, 0x3feff63da9fb3335]


def _py_cdf(logits: np.ndarray) -> np.ndarray:
    """Pure-Python restatement of codec.rs:785-798 + coder.rs:43-82 on one row (small rows only)."""
    v = len(logits)
    max_l = -math.inf
    for l in logits:
        max_l = max(max_l, float(l))
    e = [O.exp_f64(float(l) - max_l) for l in logits]
    s = 0.0
    for t in e:
        s += t
    inv_sum = 1.0 / s
    p = [float(np.float32(t * inv_sum)) for t in e]
    remaining = TOTAL - v
    sum_p = 0.0
    for t in p:
        sum_p += t
    inv = 1.0 / sum_p if sum_p > 0 else 0.0
    freqs = []
    used = 0
    for t in p:
        extra = int(t * inv * float(remaining) + 0.5)
        freqs.append(1 + extra)
        used += extra
    diff = remaining - used
    if diff:
        mi = max(range(v), key=lambda i: (freqs[i], i))   # the last of equal maxima
        freqs[mi] += diff
    return np.concatenate([[0], np.cumsum(freqs)]).astype(np.uint32)


@pytest.mark.parametrize("case", ["ref_test", "normal", "flat", "peaked", "masked", "one", "two"])
def test_oracle_cdf_matches_python_restatement(case):
    rng = np.random.default_rng(sum(map(ord, case)))
    x = {
        "ref_test": (np.arange(256, dtype=np.float32) - 128.0) * np.float32(0.1),   # codec.rs:2642
        "normal": rng.standard_normal(1500).astype(np.float32) * 3,
        "flat": np.zeros(777, np.float32),
        "peaked": np.concatenate([rng.standard_normal(999), [60.0]]).astype(np.float32),
        "masked": np.where(rng.random(600) < 0.5, -np.inf, rng.standard_normal(600)).astype(np.float32),
        "one": np.array([1.5], np.float32),
        "two": np.array([0.0, -800.0], np.float32),
    }[case]
    got = O.cdf_from_logits(x[None])[0]
    np.testing.assert_array_equal(got, _py_cdf(x))
    assert got[0] == 0 and got[-1] == TOTAL and np.all(np.diff(got.astype(np.int64)) >= 1)


def test_oracle_lookup_is_the_interval_search():
    x = np.random.default_rng(3).standard_normal(500).astype(np.float32)
    c = O.cdf_from_logits(x[None])[0]
    for cum in [0, 1, int(c[1]), int(c[100]) - 1, int(c[100]), TOTAL - 1]:
        s = O.cdf_lookup(c, cum)
        assert c[s] <= cum < c[s + 1]
    assert O.cdf_lookup(c, TOTAL) == 500


# The device kernel's summation, restated in Python: runs of terms are added as an integer sum of
# their roundings to the running sum's ulp (a tie adds the unit that leaves the sum even); a
# binade crossing or a zero / tiny running sum stops the run and that term is added by one IEEE
# addition.  (Chunk and block sizes, and the parity-map scan that parallelises the integer sum,
# do not change the arithmetic.)
def _blocked_sum(xs):
    s, i, n = 0.0, 0, len(xs)
    while i < n:
        if s == 0.0 or s < 2.0 ** -900 or s != s:
            s = s + xs[i]
            i += 1
            continue
        e = math.frexp(s)[1] - 1
        su = int(math.ldexp(s, 52 - e))
        acc, j = 0, i
        while j < n:
            t = math.ldexp(xs[j], 52 - e) if xs[j] == xs[j] else math.inf
            if not t < 2.0 ** 53:
                break
            f = math.floor(t)
            fr = t - f
            inc = int(f) + (fr > 0.5) + (fr == 0.5 and (su + acc + int(f)) % 2 == 1)
            if su + acc + inc >= 2 ** 53:
                break
            acc += inc
            j += 1
        s = math.ldexp(float(su + acc), e - 52)
        if j < n:
            s = s + xs[j]
            j += 1
        i = j
    return s


def _seq_sum(xs):
    s = 0.0
    for x in xs:
        s += x
    return s


@pytest.mark.parametrize("seed", range(6))
def test_blocked_summation_is_exactly_sequential(seed):
    rng = np.random.default_rng(seed)
    rows = [
        np.exp(rng.standard_normal(5000) * 4 - 8),                       # softmax-like terms
        rng.random(3000) * 2.0 ** -30,                                    # tiny terms
        np.concatenate([[0.0] * 50, rng.random(2000)]),                   # leading zeros
        np.concatenate([[2.0 ** -1000], rng.random(300) * 2.0 ** -990]),  # running sum below 2^-900
        np.floor(rng.random(4000) * 8) * 0.5,                             # exact multiples of 1/2
        np.concatenate([rng.random(1000), [1.0], rng.random(1000) * 1e-17]),
        np.concatenate([[2.0 ** 53], np.ones(100), [3.0] * 50, np.ones(7)]),      # a tie at every term
        np.concatenate([[1.0], [2.0 ** -53] * 1000, [3 * 2.0 ** -53] * 9, rng.random(20)]),
        np.concatenate([[0.75], [2.0 ** -54] * 300, [2.0 ** -1] * 3, [2.0 ** -53] * 300]),
    ]
    for xs in rows:
        xs = [float(v) for v in xs]
        assert _bits(_blocked_sum(xs)) == _bits(_seq_sum(xs))


def test_cdf_entry_points_reject_bad_shapes_without_a_gpu():
    from redukt_b200.plugin import PluginLibrary

    lib = PluginLibrary()
    with pytest.raises(ValueError):
        lib.cdf(np.zeros((2, 0), np.float32))
    with pytest.raises(ValueError):
        lib.cdf(np.zeros((1, 1), np.float32), symbols=np.zeros(1, np.uint32), cum_freqs=np.zeros(1, np.uint32))
    from redukt_b200.plugin import BackendResult
    assert lib.cdf_device(1, 1, 10, 9, 1, 11) == BackendResult.INVALID_ARGUMENT      # ld_logits < vocab
    assert lib.cdf_device(1, 1, 10, 10, 1, 10) == BackendResult.INVALID_ARGUMENT     # ld_cdf < vocab + 1
    assert lib.cdf_device(1, 1, TOTAL, TOTAL, 1, TOTAL + 1) == BackendResult.INVALID_ARGUMENT
    assert lib.cdf_device(1, 1, 10, 2**31, 1, 11) == BackendResult.INVALID_ARGUMENT   # int stride overflow
    assert lib.cdf_device(1, 1, 10, 10, 1, 2**32 - 1) == BackendResult.INVALID_ARGUMENT


# ----------------------------------------------------------------------------------------------
# GPU: the kernel against the oracle
# ----------------------------------------------------------------------------------------------

def _rows(v: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    rows = [
        rng.standard_normal(v) * 3,                                       # LM-like logits
        rng.standard_normal(v) * 0.01,                                    # nearly flat
        np.zeros(v),                                                      # flat: argmax ties
        np.concatenate([rng.standard_normal(v - 1), [80.0]]),             # one dominant token
        np.where(rng.random(v) < 0.3, -np.inf, rng.standard_normal(v) * 5),   # masked tokens
        -np.abs(rng.standard_normal(v)) * 400,                            # exp underflow, subnormals
        np.round(rng.standard_normal(v) * 4) / 4,                         # repeated values
        np.linspace(-30, 30, v),
    ]
    return np.stack(rows).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("vocab", [50280, 4096, 4097, 1000, 3, 1, 53248, 53249, 65536])
def test_device_cdf_bit_identical_to_oracle(vocab):
    from redukt_b200.plugin import PluginLibrary

    x = _rows(vocab, vocab)
    want = O.cdf_from_logits(x, threads=8)
    got, _ = PluginLibrary().cdf(x)
    np.testing.assert_array_equal(got, want)
    assert np.all(got[:, -1] == TOTAL)


@pytest.mark.gpu
def test_device_cdf_nan_row_matches_oracle():
    from redukt_b200.plugin import PluginLibrary

    x = np.random.default_rng(1).standard_normal((2, 3000)).astype(np.float32)
    x[0, 17] = np.nan
    x[1, :] = -np.inf
    got, _ = PluginLibrary().cdf(x)
    np.testing.assert_array_equal(got, O.cdf_from_logits(x))


@pytest.mark.gpu
def test_device_cdf_many_rows_full_vocab():
    from redukt_b200.plugin import PluginLibrary

    rng = np.random.default_rng(11)
    x = (rng.standard_normal((64, 50280)) * rng.uniform(0.5, 6, (64, 1))).astype(np.float32)
    got, _ = PluginLibrary().cdf(x)
    np.testing.assert_array_equal(got, O.cdf_from_logits(x, threads=16))


@pytest.mark.gpu
def test_encoder_and_decoder_queries():
    from redukt_b200.plugin import PluginLibrary

    lib = PluginLibrary()
    rng = np.random.default_rng(5)
    n, v = 16, 50280
    x = (rng.standard_normal((n, v)) * 3).astype(np.float32)
    want = O.cdf_from_logits(x, threads=8)
    sym = rng.integers(0, v, n).astype(np.uint32)
    sym[3] = v            # out of range
    _, q = lib.cdf(x, symbols=sym, want_cdf=False)
    for r in range(n):
        if sym[r] < v:
            assert tuple(q[r]) == (sym[r], want[r, sym[r]], want[r, sym[r] + 1])
        else:
            assert tuple(q[r]) == (v, 0xFFFFFFFF, 0xFFFFFFFF)
    cum = rng.integers(0, TOTAL, n).astype(np.uint32)
    cum[0], cum[1], cum[2] = 0, TOTAL - 1, TOTAL
    got, q = lib.cdf(x, cum_freqs=cum)
    np.testing.assert_array_equal(got, want)
    for r in range(n):
        s = O.cdf_lookup(want[r], int(cum[r]))
        if s < v:
            assert tuple(q[r]) == (s, want[r, s], want[r, s + 1])
        else:
            assert tuple(q[r]) == (v, 0xFFFFFFFF, 0xFFFFFFFF)


@pytest.mark.gpu
def test_device_entry_point_with_strides_and_stream():
    import torch

    from redukt_b200.plugin import BackendResult, PluginLibrary

    lib = PluginLibrary()
    n, v = 5, 2000
    x = _rows(v, 9)[:n]
    d_x = torch.zeros((n, v + 24), dtype=torch.float32, device="cuda")
    d_x[:, :v] = torch.from_numpy(x)
    d_c = torch.zeros((n, v + 40), dtype=torch.int64, device="cuda").view(torch.int32)   # ld = 2 (v + 40)
    ld_c = d_c.shape[1]
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    rc = lib.cdf_device(d_x.data_ptr(), n, v, v + 24, d_c.data_ptr(), ld_c, stream=stream.cuda_stream)
    assert rc == BackendResult.OK, lib.last_error()
    stream.synchronize()
    got = d_c.cpu().numpy().view(np.uint32)[:, :v + 1]
    np.testing.assert_array_equal(got, O.cdf_from_logits(x))
    assert np.all(d_c.cpu().numpy()[:, v + 1:] == 0)   # nothing written past each row
