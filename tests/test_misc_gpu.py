"""Hadamard and fp8 row-quant kernels against the oracle."""
import numpy as np
import pytest
import torch

from oracle import vq2_oracle as O

pytestmark = pytest.mark.gpu


def test_hadamard_rows():
    from vq2_vllm.kernels.vq2_kernel import had_act_batch
    g = torch.Generator().manual_seed(0)
    x = torch.randn(37, 4096, generator=g)
    y = had_act_batch(x.cuda()).cpu().numpy()
    np.testing.assert_allclose(y, O.had_act_batch(x.numpy()), rtol=1e-5, atol=1e-5)
    xb = x.bfloat16()
    yb = had_act_batch(xb.cuda())
    assert yb.dtype == torch.bfloat16
    np.testing.assert_allclose(yb.float().cpu().numpy(), O.had_act_batch(xb.float().numpy()), rtol=1e-2, atol=2e-2)
    # padding of a ragged last dim
    z = had_act_batch(torch.randn(3, 100, generator=g).cuda())
    assert z.shape == (3, 128)


def test_quant_fp8_rows_bit_exact():
    from vq2_vllm.kernels.ds4_vq2_cuda import quant_fp8_rows
    g = torch.Generator().manual_seed(1)
    x = torch.randn(300, 2048, generator=g) * torch.rand(300, 1, generator=g) * 10
    x[5] = 0.0
    q, inv = quant_fp8_rows(x.cuda())
    rq, rinv = O.quant_fp8_rows(x.numpy())
    np.testing.assert_array_equal(inv.cpu().numpy(), rinv)
    np.testing.assert_array_equal(q.float().cpu().numpy(), rq)
