"""Gated DeltaNet prefill (evie_gdn_chunk_prefill) against the oracle's token-sequential recurrence.

Tolerances: the final state within 1e-3 relative (Frobenius); outputs are bf16, so within one bf16 rounding of the
oracle's f32 output plus 1e-3 relative of the row norm."""
import numpy as np
import pytest
import torch

import oracle
from tests._inputs import bf16_bits, gdn_prefill_inputs


def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H,s0", [(1, 1, 1, False), (2, 130, 3, False), (1, 64, 2, True), (2, 257, 4, True)])
def test_prefill_matches_oracle(B, T, H, s0, cuda):
    from evie_b200 import ops

    x = gdn_prefill_inputs(B, T, H, 3, s0=s0)
    S_ref = x["S"].numpy().copy()
    o_ref = oracle.gdn_prefill(S_ref, bf16_bits(x["q"]), bf16_bits(x["k"]), bf16_bits(x["v"]), x["g"].numpy(),
                               x["beta"].numpy())
    S = x["S"].to(cuda)
    o = ops.gdn_chunk_prefill(x["q"].to(cuda), x["k"].to(cuda), x["v"].to(cuda), x["g"].to(cuda),
                              x["beta"].to(cuda), S)
    torch.cuda.synchronize()
    S_out = S.cpu().numpy()
    o_out = o.float().cpu().numpy()
    assert _rel(S_out, S_ref) < 1e-3
    err = np.abs(o_out - o_ref)
    bound = np.abs(o_ref) * 2.0 ** -8 + 1e-3 * np.linalg.norm(o_ref, axis=-1, keepdims=True) / np.sqrt(128)
    assert np.all(err <= bound), float((err - bound).max())


@pytest.mark.gpu
def test_prefill_empty_sequence_keeps_state(cuda):
    from evie_b200 import ops

    x = gdn_prefill_inputs(1, 1, 2, 5, s0=True)
    S = x["S"].to(cuda)
    S0 = S.clone()
    q = x["q"][:, :0].contiguous().to(cuda)
    ops.gdn_chunk_prefill(q, q, q, x["g"][:, :0].contiguous().to(cuda), x["beta"][:, :0].contiguous().to(cuda), S)
    torch.cuda.synchronize()
    assert torch.equal(S, S0)
