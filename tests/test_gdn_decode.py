"""Gated DeltaNet decode step: CUDA kernel (evie_gdn_decode_step) against the oracle's recur_body restatement."""
import numpy as np
import pytest
import torch

import oracle
from tests._inputs import bf16_bits, gdn_decode_inputs


def _run(B, H, seed, cuda):
    from evie_b200 import ops

    x = gdn_decode_inputs(B, H, seed)
    S_ref = x["S"].numpy().copy()
    o_ref = oracle.gdn_decode(S_ref, bf16_bits(x["q"]), bf16_bits(x["k"]), bf16_bits(x["v"]), x["g"].numpy(),
                              x["beta"].numpy())
    S = x["S"].to(cuda)
    o = ops.gdn_decode_step(x["q"].to(cuda), x["k"].to(cuda), x["v"].to(cuda), x["g"].to(cuda),
                            x["beta"].to(cuda), S)
    torch.cuda.synchronize()
    return S.cpu().numpy(), o.cpu().numpy(), S_ref, o_ref


def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("B,H", [(1, 1), (3, 5), (64, 16)])
def test_decode_step_matches_oracle(B, H, cuda):
    S, o, S_ref, o_ref = _run(B, H, 2, cuda)
    # fp32 throughout; only the summation order differs from the oracle
    assert _rel(S, S_ref) < 1e-6
    assert _rel(o, o_ref) < 1e-5
    assert np.abs(o - o_ref).max() < 1e-4


@pytest.mark.gpu
def test_decode_step_repeated_steps_track_oracle(cuda):
    """Ten steps in a row on the same state (the decode loop) stay within the DeltaNet state tolerance."""
    from evie_b200 import ops

    B, H = 4, 16
    x0 = gdn_decode_inputs(B, H, 7)
    S_ref = x0["S"].numpy().copy()
    S = x0["S"].to(cuda)
    for step in range(10):
        x = gdn_decode_inputs(B, H, 100 + step)
        o_ref = oracle.gdn_decode(S_ref, bf16_bits(x["q"]), bf16_bits(x["k"]), bf16_bits(x["v"]), x["g"].numpy(),
                                  x["beta"].numpy())
        o = ops.gdn_decode_step(x["q"].to(cuda), x["k"].to(cuda), x["v"].to(cuda), x["g"].to(cuda),
                                x["beta"].to(cuda), S)
    torch.cuda.synchronize()
    assert _rel(S.cpu().numpy(), S_ref) < 1e-3
    assert _rel(o.cpu().numpy(), o_ref) < 1e-3
