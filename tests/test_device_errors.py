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


@pytest.mark.gpu
def test_model_calls_report_a_give_up(cuda, tmp_path):
    """evie_forward and evie_decode_greedy read the device's give-up count behind their own work and return
    EVIE_ERR_TIMEOUT instead of success with incomplete outputs; the count then restarts. The give-up is made on
    purpose by the probe (a wait on a barrier nothing completes), the way a kernel of the call would count one."""
    from evie_b200 import EvieError, checkpoint as ck, ops
    from evie_b200.gpu import GpuModel, GpuSeq

    path = str(tmp_path / "tiny")
    ck.write_checkpoint(path, ck.tiny_config(vocab_size=512, num_hidden_layers=4), seed=0)
    m = GpuModel(path, max_ctx=128, slots=1, max_rows=16)
    toks = np.arange(3, 11, dtype=np.uint32)
    ops.poll_device_errors()
    first = m.forward([GpuSeq(0, 0, toks)]).logits.copy()
    assert ops.bounded_wait_probe(10_000_000) == 1
    with pytest.raises(EvieError, match="gave up a bounded device-side wait") as e:
        m.forward([GpuSeq(0, 8, toks[:1])])
    assert e.value.status == 5
    m.reset_slot(0)
    again = m.forward([GpuSeq(0, 0, toks)]).logits  # the count restarted and the context still works
    assert np.array_equal(again, first)
    assert ops.bounded_wait_probe(10_000_000) == 1
    with pytest.raises(EvieError) as e:
        m.decode_greedy([GpuSeq(0, 8, toks[:1])], 2)
    assert e.value.status == 5
    ops.poll_device_errors()
    m.close()
