"""Native Q8 payload files (.rbin flag bit 6): the Q8 matrices stored as int8 + group scales, so the
engine loads them without reading f32 weights or quantising.  The converter must reproduce the
reference's quantisation recipe exactly (the oracle's restatement of Q8wMatrix::quantize), and a
payload file must run bit-identically to the same model quantised at load."""
import os

import numpy as np
import pytest

from conftest import q8, shared_backend
from oracle import oracle as O
from redukt_b200 import rbin
from redukt_b200.workload import zipf_tokens


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.fixture(scope="module")
def payload_pair(small_gauss_rbin, model_dir):
    dst = os.path.join(model_dir, "gauss_small.q8payload.rbin")
    rbin.to_q8_payload(small_gauss_rbin, dst)
    return small_gauss_rbin, dst


def test_converter_matches_the_reference_recipe(payload_pair):
    src, dst = payload_pair
    dims, flags, arrays = rbin.read_arrays(src)
    pdims, pflags, payload = rbin.read_q8_payload(dst)
    assert pdims == dims and pflags == flags | rbin.FLAG_Q8 | rbin.FLAG_Q8_PAYLOAD
    for name, a in arrays.items():
        if rbin.is_q8_matrix(name):
            q, s = payload[name]
            q_ref, s_ref = O.q8_quantize(a, 64)
            assert np.array_equal(q, q_ref) and np.array_equal(bits(s), bits(s_ref)), name
        else:
            assert np.array_equal(bits(payload[name]), bits(a)), name


def test_payload_file_size_and_flags(payload_pair, tmp_path):
    src, dst = payload_pair
    dims, flags, _ = rbin.read_header(src)
    n_f32 = sum(int(np.prod(s)) for n, s in rbin.array_order(dims, flags) if not rbin.is_q8_matrix(n))
    n_q8 = sum(int(np.prod(s)) for n, s in rbin.array_order(dims, flags) if rbin.is_q8_matrix(n))
    assert os.path.getsize(dst) == rbin.RBIN_HEADER.size + 4 * n_f32 + n_q8 + 4 * (n_q8 // 64)
    with pytest.raises(ValueError):
        rbin.read_arrays(dst)          # not an f32 body
    with pytest.raises(ValueError):
        rbin.to_q8_payload(dst, str(tmp_path / "again.rbin"))
    with pytest.raises(ValueError):
        rbin.with_flags(src, str(tmp_path / "bad.rbin"), rbin.FLAG_Q8_PAYLOAD)


@pytest.mark.gpu
def test_payload_loads_bit_identical_to_quantise_on_load(payload_pair):
    src, dst = payload_pair
    V = None
    outs, mats = {}, {}
    for name, path in (("load", q8(src)), ("payload", dst)):
        b = shared_backend(path)
        V = b.vocab_size
        mats[name] = [b.get_q8(w, layer) for w, layer in (("emb", 0), ("in_proj", 0), ("out_proj", 2))]
        n = 5
        toks = zipf_tokens(n, 4, vocab=V, seed_base=3)
        b.batch_init(n)
        outs[name] = np.stack([b.forward_batch(list(range(n)), toks[:, t]).copy() for t in range(4)], 1)
    for (qa, sa), (qb, sb) in zip(mats["load"], mats["payload"]):
        assert np.array_equal(qa, qb) and np.array_equal(bits(sa), bits(sb))
    assert np.array_equal(bits(outs["load"]), bits(outs["payload"]))
