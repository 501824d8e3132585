"""K3 moe_align parity: bit-exact against the reference's deterministic torch align (golden
fixtures) and the numpy oracle, including multi-chunk sizes."""
import numpy as np
import pytest
import torch

from golden_io import load_align
from oracle import vq2_oracle as O

pytestmark = pytest.mark.gpu


def _align():
    from vq2_vllm.kernels.moe_align import moe_align
    return moe_align


def _cmp(got, want):
    st, ss, val, be, nb = got
    wst, wss, wval, wbe, wnb = want
    assert nb == wnb
    assert np.array_equal(st.cpu().numpy(), wst) and np.array_equal(ss.cpu().numpy(), wss)
    assert np.array_equal(val.cpu().numpy(), wval) and np.array_equal(be.cpu().numpy(), wbe)


def test_golden_cases():
    for ids, E, BM, nblk, st, ss, val, be in load_align():
        t = torch.from_numpy(ids).cuda()
        _cmp(_align()(t, E, BM), (st, ss, val, be, nblk))
        _cmp(_align()(t.long(), E, BM), (st, ss, val, be, nblk))


@pytest.mark.parametrize("N,k,E,BM", [(8192, 8, 256, 64), (8192, 8, 256, 128), (65536, 8, 256, 128),
                                      (3000, 6, 1000, 16), (1, 1, 1, 1)])
def test_large_vs_oracle(N, k, E, BM):
    from vq2_vllm import synth
    ids, _ = synth.route_zipf(N, E, k, seed=N + E) if k <= E else (None, None)
    t = ids.cuda()
    _cmp(_align()(t, E, BM), O.moe_align(ids.numpy(), E, BM))


def test_out_of_range_ids_are_clamped():
    ids = torch.tensor([[0, 9], [-3, 2], [7, 100]], dtype=torch.int32)
    got = _align()(ids.cuda(), 8, 4)
    _cmp(got, O.moe_align(ids.clamp(0, 7).numpy(), 8, 4))
