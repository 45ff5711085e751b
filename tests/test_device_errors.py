"""The failure path of the kernels' bounded device-side waits (every mbarrier wait gives up after a deadline of
%globaltimer, counts the give-up and lets the kernel drain and return): a wait on a barrier that nothing completes
gives up, evie_poll_device_errors reports it once with EVIE_ERR_TIMEOUT, and the device keeps working."""
import numpy as np
import pytest

import oracle
from tests._inputs import bf16_bits, gdn_decode_inputs


@pytest.mark.gpu
def test_bounded_wait_gives_up_and_is_reported_once(cuda):
    from evie_b200 import EvieError, ops

    ops.poll_device_errors()  # nothing pending before the probe
    assert ops.bounded_wait_probe(10_000_000) == 1  # 10 ms on a barrier with no arrivals
    with pytest.raises(EvieError, match="gave up a bounded device-side wait") as e:
        ops.poll_device_errors()
    assert e.value.status == 5  # EVIE_ERR_TIMEOUT
    ops.poll_device_errors()  # the count restarted

    # the context is still usable: a decode step after the probe matches the oracle
    x = gdn_decode_inputs(2, 2, 2)
    S_ref = x["S"].numpy().copy()
    o_ref = oracle.gdn_decode(S_ref, bf16_bits(x["q"]), bf16_bits(x["k"]), bf16_bits(x["v"]), x["g"].numpy(),
                              x["beta"].numpy())
    S = x["S"].to(cuda)
    o = ops.gdn_decode_step(x["q"].to(cuda), x["k"].to(cuda), x["v"].to(cuda), x["g"].to(cuda),
                            x["beta"].to(cuda), S)
    ops.poll_device_errors()
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))
    assert rel(S.cpu().numpy(), S_ref) < 1e-6  # the decode step's own bars (fp32, summation order only)
    assert rel(o.cpu().numpy(), o_ref) < 1e-5


def test_probe_rejects_limits_above_the_kernels_deadline():
    """Argument checks run before any device work, so they hold without a GPU."""
    from evie_b200 import EvieError, lib, ops

    lib()
    with pytest.raises(EvieError, match="limit above"):
        ops.bounded_wait_probe(3_000_000_000)
