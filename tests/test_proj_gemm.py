"""Projection GEMM (evie_proj_gemm, the tcgen05 kernel behind every projection and the LM head) against evie-core's
`matmul` arithmetic (the oracle's restatement of kernels.rs:138-268) and a float64 product.

The operand is an f32 matrix split into bf16 planes hi + lo; the planes the kernel returns are K slices whose sum is
the product. Shapes cover the decode tiles (R = 1, 64, 100: 16-, 64- and 128-row operand tiles, K cut into slices),
partial weight tiles, and the persistent prefill tiles (several tiles per CTA, partial R and M tiles)."""
import numpy as np
import pytest
import torch

import oracle
from tests._inputs import bf16_bits


def _case(M, K, R, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(M, K, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(R, K, generator=g)
    return w, x


def _run(w, x, cuda, max_planes=16):
    from evie_b200 import ops

    x2 = ops.split_planes(x.to(cuda))
    y = ops.proj_gemm(w.to(cuda), x2, max_planes)
    torch.cuda.synchronize()
    planes = y.shape[0]
    tot = y[0].clone()
    for p in range(1, planes):
        tot += y[p]
    return tot.cpu().numpy(), planes


def _scale(w, x):
    return float((w.float().abs().double() @ x.abs().double().T).max())


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,R", [(300, 256, 1), (2560, 4096, 64), (1000, 512, 100), (640, 576, 300)])
def test_matches_oracle_matmul(M, K, R, cuda):
    w, x = _case(M, K, R, 11 + M + R)
    y, planes = _run(w, x, cuda)
    ref = oracle.matmul(bf16_bits(w).reshape(M, K), x.numpy())
    err = np.abs(y - ref).max() / _scale(w, x)
    assert err < 1e-5, (err, planes)


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,R", [(12352, 2560, 64), (2560, 9216, 64), (40000, 1024, 64), (1536, 2560, 4096),
                                   (8224, 1024, 7), (18432, 2560, 128)])
def test_matches_float64(M, K, R, cuda):
    w, x = _case(M, K, R, 5 + K + R)
    y, planes = _run(w, x, cuda)
    ref = (x.double() @ w.double().T).numpy()
    err = np.abs(y - ref).max() / _scale(w, x)
    assert err < 2e-6, (err, planes)
    if R <= 128:
        assert planes >= 1
    else:
        assert planes == 1


@pytest.mark.gpu
def test_slices_sum_to_one_slice(cuda):
    """The K-sliced planes add up to the single-slice product (the consumers' split-K reduction)."""
    w, x = _case(2560, 4096, 64, 3)
    y1, p1 = _run(w, x, cuda, max_planes=1)
    yk, pk = _run(w, x, cuda, max_planes=16)
    assert p1 == 1 and pk > 1
    # the two differ only in the order of the f32 accumulation (tensor-core sums per 16-element step)
    assert np.abs(y1 - yk).max() / _scale(w, x) < 2e-6
