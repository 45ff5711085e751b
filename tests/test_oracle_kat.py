"""The CPU oracle pinned to the known-answer tests of evie-core's own unit tests.

crates/evie-core/src/kernels.rs:697-718 (matmul_matches_reference, topk_and_rank) and
crates/evie-core/src/steering.rs:257-294 (add_mul_set, gate_latches_and_is_causal), restated on the oracle.
"""
import numpy as np

import oracle


def _xorshift_mat(rows, cols, seed):
    """kernels.rs:674-685: xorshift64 uniform(-1, 1) values stored as bf16 (truncated f32 bits)."""
    s = np.uint64(seed)
    out = np.empty(rows * cols, np.uint16)
    M = np.uint64(0xFFFFFFFFFFFFFFFF)
    for i in range(rows * cols):
        s ^= (s << np.uint64(13)) & M
        s ^= s >> np.uint64(7)
        s ^= (s << np.uint64(17)) & M
        f = np.float32(np.float32(int(s >> np.uint64(11))) / np.float32(2.0 ** 53)) * np.float32(2.0) - np.float32(1.0)
        out[i] = np.uint16(np.array([f], np.float32).view(np.uint32)[0] >> 16)
    return out.reshape(rows, cols)


def _bf(u16):
    return (u16.astype(np.uint32) << 16).view(np.float32)


def test_matmul_matches_reference():
    # every dispatch path: n == 1 (dot_rows), 2..7 (multi_dot), >= 8 (packed GEMM), tails not multiple of 8/16
    for rows, cols in [(37, 29), (64, 256), (48, 520), (33, 1000)]:
        w = _xorshift_mat(rows, cols, rows * 31 + cols)
        wf = _bf(w).astype(np.float64)
        for n in [1, 2, 3, 5, 7, 8, 13, 50]:
            x = _bf(_xorshift_mat(n, cols, 7 + n))
            y = oracle.matmul(w, x)
            ref = (x.astype(np.float64) @ wf.T).astype(np.float32)
            assert np.all(np.abs(y - ref) < 1e-3 * (1.0 + np.abs(ref))), (rows, cols, n)


def test_topk_and_rank():
    v = np.array([0.5, 3.0, -1.0, 2.0, 2.5], np.float32)
    idx, _ = oracle.topk(v, 3)
    assert list(idx) == [1, 4, 3]
    assert int((v > v[3]).sum()) == 2  # rank_of(values, 3)


def test_topk_ties_first_index_wins():
    v = np.array([1.0, 5.0, 5.0, 2.0, 5.0], np.float32)
    idx, _ = oracle.topk(v, 2)
    assert list(idx) == [1, 2]
    assert oracle.greedy(v) == 1


def test_steering_add_mul_set():
    ivs = [
        dict(layer=0, neuron=1, mode="add", value=2.0),
        dict(layer=0, neuron=2, mode="mul", value=0.0),
        dict(layer=1, neuron=0, mode="set", value=7.0),
    ]
    plan = oracle.compile_plan(ivs, 2, 3, lambda l, n: 0.5)
    st = oracle.GateState()
    plan.begin(st, 2)
    a = np.array([1, 1, 1, 2, 2, 2], np.float32)
    plan.apply(0, a, 3, st)
    assert a.tolist() == [1.0, 2.0, 0.0, 2.0, 3.0, 0.0]
    b = np.array([1, 1, 1], np.float32)
    plan.apply(1, b, 3, st)
    assert b.tolist() == [7.0, 1.0, 1.0]


def test_gate_latches_and_is_causal():
    iv = dict(layer=0, neuron=0, mode="add", value=1.0,
              gate=dict(detectors=[dict(layer=1, neuron=0, weight=1.0)], threshold=5.0))
    plan = oracle.compile_plan([iv], 2, 1, lambda l, n: 1.0)
    st = oracle.GateState()
    plan.begin(st, 2)
    l0 = np.array([0, 0], np.float32)
    plan.apply(0, l0, 1, st)
    assert l0.tolist() == [0.0, 0.0]
    l1 = np.array([1, 9], np.float32)
    plan.apply(1, l1, 1, st)
    assert st.open(0)
    plan.begin(st, 1)
    l0 = np.array([0], np.float32)
    plan.apply(0, l0, 1, st)
    assert l0.tolist() == [1.0]


def test_compand_matches_capture_rule():
    # worker.rs:97-112: q = round(127 sqrt(min(|v|, 1))) with the sign of v; Trace::decode inverts it
    for v, q in [(0.0, 0), (1.0, 127), (-1.0, -127), (2.0, 127), (0.25, 64), (-0.25, -64), (1e-6, 0)]:
        assert oracle.compand(v) == q
