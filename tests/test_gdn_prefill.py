"""Gated DeltaNet prefill against the oracle's token-sequential recurrence: the chunked tensor-core kernel
(evie_gdn_chunk_prefill) and the token-by-token kernel (evie_gdn_prefill_tokenwise).

Tolerances: the final state within 1e-3 relative (Frobenius); outputs are bf16, so within one bf16 rounding of the
oracle's f32 output plus 1e-3 relative of the row norm. Cases cover a single token, ragged last chunks, several
sequences and heads, a non-zero entering state, an empty prompt and the full benchmark size (B=8, T=8192, H=16),
whose heads are checked against the oracle on a sample."""
import numpy as np
import pytest
import torch

import oracle
from tests._inputs import bf16_bits, gdn_prefill_inputs


def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _check(S_out, S_ref, o_out, o_ref):
    assert _rel(S_out, S_ref) < 1e-3, _rel(S_out, S_ref)
    err = np.abs(o_out - o_ref)
    bound = np.abs(o_ref) * 2.0 ** -8 + 1e-3 * np.linalg.norm(o_ref, axis=-1, keepdims=True) / np.sqrt(128)
    assert np.all(err <= bound), float((err - bound).max())


def _impl(name):
    from evie_b200 import ops

    return {"chunk": ops.gdn_chunk_prefill, "tokenwise": ops.gdn_prefill_tokenwise}[name]


@pytest.mark.gpu
@pytest.mark.parametrize("impl", ["chunk", "tokenwise"])
@pytest.mark.parametrize("B,T,H,s0", [(1, 1, 1, False), (2, 130, 3, False), (1, 64, 2, True), (2, 257, 4, True),
                                      (3, 1000, 2, True), (1, 63, 1, True)])
def test_prefill_matches_oracle(B, T, H, s0, impl, cuda):
    from evie_b200 import ops

    x = gdn_prefill_inputs(B, T, H, 3, s0=s0)
    S_ref = x["S"].numpy().copy()
    o_ref = oracle.gdn_prefill(S_ref, bf16_bits(x["q"]), bf16_bits(x["k"]), bf16_bits(x["v"]), x["g"].numpy(),
                               x["beta"].numpy())
    S = x["S"].to(cuda)
    o = _impl(impl)(x["q"].to(cuda), x["k"].to(cuda), x["v"].to(cuda), x["g"].to(cuda), x["beta"].to(cuda), S)
    ops.poll_device_errors()
    _check(S.cpu().numpy(), S_ref, o.float().cpu().numpy(), o_ref)


@pytest.mark.gpu
def test_prefill_b8_t8192_h16_sampled_heads(cuda):
    """B=8, T=8192, H=16 (S0 = 0) through the chunked kernel; four (sequence, head) pairs against the
    oracle over the whole 8192-token sequence."""
    from evie_b200 import ops

    B, T, H = 8, 8192, 16
    x = gdn_prefill_inputs(B, T, H, 3)
    S = x["S"].to(cuda)
    o = ops.gdn_chunk_prefill(x["q"].to(cuda), x["k"].to(cuda), x["v"].to(cuda), x["g"].to(cuda),
                              x["beta"].to(cuda), S)
    ops.poll_device_errors()
    S_out, o_out = S.cpu().numpy(), o.float().cpu().numpy()
    for b, h in [(0, 0), (3, 7), (5, 12), (7, 15)]:
        sl = lambda t: t[b:b + 1, :, h:h + 1].contiguous()  # noqa: E731
        S_ref = x["S"][b:b + 1, h:h + 1].numpy().copy()
        o_ref = oracle.gdn_prefill(S_ref, bf16_bits(sl(x["q"])), bf16_bits(sl(x["k"])), bf16_bits(sl(x["v"])),
                                   sl(x["g"]).numpy(), sl(x["beta"]).numpy())
        _check(S_out[b:b + 1, h:h + 1], S_ref, o_out[b:b + 1, :, h:h + 1], o_ref)


@pytest.mark.gpu
@pytest.mark.parametrize("impl", ["chunk", "tokenwise"])
def test_prefill_empty_sequence_keeps_state(impl, cuda):
    x = gdn_prefill_inputs(1, 1, 2, 5, s0=True)
    S = x["S"].to(cuda)
    S0 = S.clone()
    q = x["q"][:, :0].contiguous().to(cuda)
    _impl(impl)(q, q, q, x["g"][:, :0].contiguous().to(cuda), x["beta"][:, :0].contiguous().to(cuda), S)
    torch.cuda.synchronize()
    assert torch.equal(S, S0)
