"""Size-independent properties of the CPU oracle (test infrastructure), checked on random cases:
the 10-bit index format round-trips, the group Hadamard is an involution, moe_align's output is a
stable, padded, complete grouping of the pairs, the e4m3 rounding is idempotent and monotone, and
the MoE is linear in the routing weights."""
import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import vq2_oracle as O

SET = settings(max_examples=25, deadline=None)


@SET
@given(rows=st.integers(1, 6), nsub4=st.integers(1, 16), seed=st.integers(0, 2**31 - 1))
def test_pack10_round_trip(rows, nsub4, seed):
    ids = np.random.default_rng(seed).integers(0, 1024, size=(rows, 4 * nsub4))
    lo, hi = O.pack10(ids)
    assert lo.shape == ids.shape and hi.shape == (rows, nsub4)
    assert np.array_equal(O.unpack10(lo, hi), ids)


@SET
@given(n=st.integers(1, 5), groups=st.integers(1, 4), seed=st.integers(0, 2**31 - 1))
def test_hadamard_is_an_involution(n, groups, seed):
    x = np.random.default_rng(seed).standard_normal((n, 64 * groups)).astype(np.float32)
    y = O.had_act_batch(O.had_act_batch(x))
    assert np.allclose(y, x, atol=1e-5)
    h = O.hadamard(64)
    assert np.allclose(h @ h.T, np.eye(64), atol=1e-6)


@SET
@given(N=st.integers(1, 40), k=st.integers(1, 4), E=st.integers(1, 12), BM=st.sampled_from([4, 16, 64]),
       seed=st.integers(0, 2**31 - 1))
def test_moe_align_invariants(N, k, E, BM, seed):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.permutation(max(E, k))[:k] % E for _ in range(N)])
    st_, ss, val, be, nblk = O.moe_align(ids, E, BM)
    M = N * k
    assert st_.size == M + min(M, E) * BM and nblk == st_.size // BM
    pos = np.nonzero(val)[0]
    pairs = st_[pos] * k + ss[pos]
    assert np.array_equal(np.sort(pairs), np.arange(M))              # every pair exactly once
    experts = ids.reshape(-1)[pairs]
    assert np.all(np.diff(experts) >= 0)                             # grouped by expert, in order
    for e in np.unique(experts):
        sel = pairs[experts == e]
        assert np.all(np.diff(sel) > 0)                              # stable within an expert
        first = pos[experts == e][0]
        assert first % BM == 0                                       # each run starts on a block
        assert np.all(be[pos[experts == e] // BM] == e)              # blocks map to their expert


@SET
@given(seed=st.integers(0, 2**31 - 1), scale=st.floats(1e-3, 400.0))
def test_e4m3_rounding_properties(seed, scale):
    v = (np.random.default_rng(seed).standard_normal(256) * scale).astype(np.float32)
    v = np.clip(v, -448.0, 448.0)
    q = O.to_e4m3(v)
    assert np.array_equal(O.to_e4m3(q), q)                           # idempotent
    order = np.argsort(v, kind="stable")
    assert np.all(np.diff(q[order]) >= 0)                            # monotone
    a = np.abs(v.astype(np.float64))
    step = np.exp2(np.maximum(np.floor(np.log2(np.where(a > 0, a, 1.0))), -6.0) - 3.0)
    assert np.all(np.abs(q - v) <= step / 2 + 1e-12)                 # within half a step


@SET
@given(seed=st.integers(0, 2**31 - 1), a=st.floats(-2.0, 2.0), b=st.floats(-2.0, 2.0))
def test_moe_is_linear_in_routing_weights(seed, a, b):
    rng = np.random.default_rng(seed)
    E, H, I, N, k = 4, 128, 64, 3, 2
    ids = np.stack([rng.permutation(E)[:k] for _ in range(N)])
    lo13, hi13 = O.pack10(rng.integers(0, 1024, size=(E, 2 * I, H // 4)))
    lo2, hi2 = O.pack10(rng.integers(0, 1024, size=(E, H, I // 4)))
    cb = (rng.standard_normal((1024, 4)) * 0.02).astype(np.float16)
    sc13 = rng.uniform(0.5, 1.5, size=(E, 2 * I, H // 64)).astype(np.float16)
    sc2 = rng.uniform(0.5, 1.5, size=(E, H, I // 64)).astype(np.float16)
    w13, w2 = (cb, lo13, hi13, sc13), (cb, lo2, hi2, sc2)
    x = rng.standard_normal((N, H)).astype(np.float32)
    w1 = rng.uniform(0, 1, size=(N, k)).astype(np.float32)
    w2_ = rng.uniform(0, 1, size=(N, k)).astype(np.float32)
    lhs = O.moe_ref(x, ids, (a * w1 + b * w2_).astype(np.float32), w13, w2)
    rhs = a * O.moe_ref(x, ids, w1, w13, w2) + b * O.moe_ref(x, ids, w2_, w13, w2)
    assert np.allclose(lhs, rhs, rtol=1e-4, atol=1e-6 * (1 + np.abs(rhs).max()))
