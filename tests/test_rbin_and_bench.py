"""The .rbin container, the seeded models and the benchmark's byte accounting."""
import os

import numpy as np

import bench
from redukt_b200 import rbin
from redukt_b200.workload import zipf_tokens


def test_header_roundtrip_and_array_order(tmp_path):
    dims = rbin.MambaDims(vocab=300, d_model=64, n_layer=2)
    p = rbin.ensure_model(str(tmp_path / "m.rbin"), dims, kind="gaussian", seed=3,
                          flags=rbin.FLAG_NORM_BIAS | rbin.FLAG_UNTIED_HEAD)
    d2, flags, tok = rbin.read_header(p)
    assert d2 == dims and flags == rbin.FLAG_NORM_BIAS | rbin.FLAG_UNTIED_HEAD and tok == rbin.TOK_BPE
    _, _, arrays = rbin.read_arrays(p)
    names = [n for n, _ in rbin.array_order(dims, flags)]
    assert list(arrays) == names
    assert names[0] == "embeddings" and names[-1] == "lm_head_w"
    assert np.all(arrays["layers.0.A_log"][5] == np.log(np.arange(1, 17)).astype(np.float32))
    assert np.all(arrays["layers.1.D"] == 1.0) and np.all(arrays["norm_f_b"] == 0.0)
    q = rbin.with_flags(p, str(tmp_path / "m.q8.rbin"), rbin.FLAG_Q8)
    assert rbin.read_header(q)[1] & rbin.FLAG_Q8
    assert os.path.getsize(q) == os.path.getsize(p)


def test_dt_bias_is_softplus_inverse_of_log_uniform(tmp_path):
    dims = rbin.MambaDims(vocab=100, d_model=64, n_layer=1)
    p = rbin.ensure_model(str(tmp_path / "m.rbin"), dims, kind="gaussian", seed=4)
    _, _, a = rbin.read_arrays(p)
    u = np.log1p(np.exp(a["layers.0.dt_proj_b"].astype(np.float64)))
    assert u.min() >= 1e-3 * 0.999 and u.max() <= 0.1 * 1.001


def test_reference_synthetic_model_is_deterministic():
    a = list(rbin.reference_test_arrays(rbin.REFERENCE_TEST_DIMS))
    assert a[0][0] == "embeddings" and a[0][1].shape == (1200, 64)
    b = list(rbin.reference_test_arrays(rbin.REFERENCE_TEST_DIMS))
    assert all(np.array_equal(x[1], y[1]) for x, y in zip(a, b))


def test_zipf_tokens_seeded_and_in_range():
    t = zipf_tokens(3, 1000, vocab=50280)
    assert t.shape == (3, 1000) and t.max() < 50280
    assert np.array_equal(t, zipf_tokens(3, 1000, vocab=50280))
    assert not np.array_equal(t[0], t[1])
    assert np.mean(t == 0) > 0.05  # rank 1 is the most frequent id


def test_algorithmic_bytes_match_the_published_accounting():
    w_q8, s_q8 = bench.dims_bytes(rbin.MAMBA_130M, "q8")
    w_f32, s_f32 = bench.dims_bytes(rbin.MAMBA_130M, "f32")
    assert w_q8 == 153_614_208
    assert w_f32 == 516_541_440
    assert s_f32 == 5_807_520
    assert rbin.MAMBA_130M.state_bytes() == 2_801_664
