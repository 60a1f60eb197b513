"""Host restatements of two identities the packed-pipe kernels rely on (no GPU needed).

1. lane_expf2 (rk_math.cuh) scales both halves of a pair by 2^n with one 64-bit subtract and
   shift of the magic-sum bits instead of two 32-bit ones: for every argument the clamp admits,
   the pair trick gives each half exactly cephes_exp_core's scale factor.
2. k_gemv_f32_p (rk_kernels.cuh) reduces a warp's 32 outputs with a reduce-scatter over the xor
   butterfly 16, 8, 4, 2, 1.  Every output is summed by the same tree as warp_allsum, so the
   float32 results are identical, and lane l ends holding output l.

Both are checked with numpy float32 arithmetic (each operation correctly rounded, as __fadd_rn).
"""
import numpy as np

F = np.float32
EXP_LO, EXP_HI = F(-87.3365447505531), F(88.3762626647949)


def magic_bits(x):
    """bits of fx + 1.5 * 2^23, fx = x * log2(e) (cephes_exp_core's rounding step)."""
    fx = (x.astype(F) * F(1.44269504088896341)).astype(F)
    return (fx + F(12582912.0)).astype(F).view(np.uint32)


def test_pair_exponent_scale_matches_per_lane_scale():
    rng = np.random.default_rng(3)
    x = np.concatenate([np.linspace(EXP_LO, EXP_HI, 200001, dtype=F),
                        rng.uniform(EXP_LO, EXP_HI, 200000).astype(F), np.array([EXP_LO, EXP_HI, 0, -0.0], F)])
    if len(x) % 2:
        x = x[:-1]
    bits = magic_bits(x).astype(np.uint64)
    # per lane: ((bits - 0x4B400000) + 127) << 23, as cephes_exp_core computes it
    n = bits.astype(np.int64) - 0x4B400000
    assert n.min() >= -126 and n.max() <= 128
    lane = ((n + 127).astype(np.uint64) << np.uint64(23)) & np.uint64(0xFFFFFFFF)
    # pair: one 64-bit subtract of 0x4B3FFF81 in each half, one 64-bit shift by 23
    pair = bits[0::2] | (bits[1::2] << np.uint64(32))
    scaled = (pair - np.uint64(0x4B3FFF814B3FFF81)) << np.uint64(23)
    lo = scaled & np.uint64(0xFFFFFFFF)
    hi = scaled >> np.uint64(32)
    assert np.array_equal(lo, lane[0::2]) and np.array_equal(hi, lane[1::2])


def warp_allsum(vals):
    """vals [32 lanes] of one output: the butterfly every lane ends with (offsets 16..1)."""
    v = vals.astype(F).copy()
    for d in (16, 8, 4, 2, 1):
        v = (v + v[np.arange(32) ^ d]).astype(F)
    assert np.all(v == v[0]) or np.all(np.isnan(v))
    return v[0]


def reduce_scatter(vals, outputs):
    """vals [32 lanes][outputs]: k_gemv_f32_p's reduction; returns what each lane ends holding."""
    lanes = np.arange(32)
    v = [vals[l].astype(F).copy() for l in lanes]
    L = outputs
    for d in (16, 8, 4, 2, 1):
        if L > 1:
            new = []
            for l in lanes:
                p = l ^ d
                up = (l & d) != 0
                keep = v[l][L // 2:L] if up else v[l][:L // 2]
                recv = v[p][L // 2:L] if up else v[p][:L // 2]  # the partner gives away the half l keeps
                new.append((keep + recv).astype(F))
            v = new
            L //= 2
        else:
            v = [np.array([F(v[l][0] + v[l ^ d][0])]) for l in lanes]
    return np.array([x[0] for x in v], F)


def test_reduce_scatter_equals_allsum_tree():
    rng = np.random.default_rng(11)
    for outputs in (32, 16):
        for trial in range(20):
            scale = 10.0 ** rng.uniform(-3, 3)
            vals = (rng.standard_normal((32, outputs)) * scale).astype(F)
            got = reduce_scatter(vals, outputs)
            per = 32 // outputs
            for lane in range(32):
                j = lane // per
                assert got[lane].view(np.uint32) == warp_allsum(vals[:, j]).view(np.uint32), (outputs, lane)
