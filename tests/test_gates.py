"""Latching detector gates on the device (evie_set_plan / evie_gate_state / evie_reset_gates) against the oracle's
restatement of Plan::apply (crates/evie-core/src/steering.rs:150-210) driving the same small model.

The gates are checked where the reference's rules differ from each other:
  - a gated op before the deciding layer takes effect from the next call on (steering.rs:194-197);
  - a gated op at or after the deciding layer applies from the trigger row on within the call;
  - a gate whose detectors are all out of range decides at layer 0 on a zero sum (steering.rs:129-133);
  - a gate that never fires; an ungated op beside gated ones; a second slot without gates in the same batch;
  - the latch across calls, the score on the last row, and evie_reset_gates.
Thresholds are placed at the midpoint of a wide gap in the oracle's detector sums, so that the ~1e-5 relative
difference between the device's and the oracle's activations cannot move the trigger row."""
import os

import numpy as np
import pytest

import oracle
from evie_b200 import checkpoint as ck
from evie_b200.steering import Detector, Gate, Intervention, Plan

LOGIT_TOL = 2e-3  # f32 KV cache, as the full-model tests
SCALE = 0.5
NEVER = 1e30


@pytest.fixture(scope="module")
def gate_ckpt(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("gckpt") / "tiny")
    ck.write_checkpoint(path, ck.tiny_config(vocab_size=2048, num_hidden_layers=8), seed=0)
    return path


@pytest.fixture(scope="module")
def gate_ref(gate_ckpt):
    return oracle.Model(gate_ckpt)


DETS = [Detector(3, 11, 1.0), Detector(5, 40, -0.5)]


def _interventions(thr: float):
    return [
        Intervention(1, 9, 0.8, "add", gate=Gate(list(DETS), thr)),        # before the deciding layer (5)
        Intervention(5, 3, 2.5, "set", gate=Gate(list(DETS), thr)),        # at the deciding layer
        Intervention(7, 20, -3.0, "mul", gate=Gate(list(DETS), thr)),      # after it
        Intervention(2, 5, 0.3, "add"),                                     # ungated
        Intervention(6, 12, 0.5, "add", gate=Gate([Detector(99, 1)], -1.0)),  # no detector in range: decides at 0
        Intervention(4, 1, 9.0, "set", gate=Gate(list(DETS), NEVER)),      # never opens
    ]


def _oracle_plan(ivs, cfg):
    d = []
    for iv in ivs:
        x = dict(layer=iv.layer, neuron=iv.neuron, mode=iv.mode, value=iv.value)
        if iv.gate is not None:
            x["gate"] = dict(detectors=[dict(layer=t.layer, neuron=t.neuron, weight=t.weight) for t in iv.gate.detectors],
                             threshold=iv.gate.threshold)
        d.append(x)
    return oracle.compile_plan(d, cfg.n_layers, cfg.intermediate, lambda l, n: 1.0)


def _gpu(path, **kw):
    from evie_b200.gpu import GpuModel

    old = os.environ.get("EVIE_KV_F32")
    os.environ["EVIE_KV_F32"] = "1"
    try:
        return GpuModel(path, **kw)
    finally:
        if old is None:
            del os.environ["EVIE_KV_F32"]
        else:
            os.environ["EVIE_KV_F32"] = old


def _calibrate(ref, prompt):
    """Runs the plan with the detector gates held shut; returns (trigger row, threshold) at the widest record gap
    of the detector sum. Ops at or after the deciding layer only touch rows from the trigger on, which cannot
    change the sums of earlier rows or the trigger row's own sum, so the open run sees the same sums up to it."""
    cfg = ref.cfg
    plan = _oracle_plan(_interventions(NEVER), cfg)
    st = oracle.GateState()
    ref.forward([dict(cache=ref.new_cache(), tokens=prompt, plan=plan, gate=st)])
    p = st.partial(0)
    best = None
    for t in range(3, len(p)):
        gap = p[t] - p[:t].max()
        if gap > 0 and (best is None or gap > best[0]):
            best = (gap, t)
    assert best is not None and best[0] > 0.05, "no usable gap in the detector sums"
    gap, t = best
    return t, float(np.float32(p[:t].max() + gap / 2))


@pytest.mark.gpu
def test_gates_match_oracle_across_calls(gate_ckpt, gate_ref, cuda):
    from evie_b200.gpu import GpuSeq

    ref = gate_ref
    cfg = ref.cfg
    L, n = cfg.n_layers, cfg.intermediate
    rng = np.random.default_rng(7)
    prompt = rng.integers(0, 2048, 40).astype(np.uint32)
    other = rng.integers(0, 2048, 12).astype(np.uint32)
    t, thr = _calibrate(ref, prompt)
    ivs = _interventions(thr)

    m = _gpu(gate_ckpt, max_ctx=256, slots=2, max_rows=64)
    scale = np.full(L * n, SCALE, np.float32)
    m.set_scale(scale)
    # a decode-shaped call captured before any gate exists; setting the plan must drop that graph
    m.forward([GpuSeq(1, 0, other[:1])])
    m.reset_slot(1)
    m.set_plan(0, Plan.compile(ivs, L, n, lambda l, nn: 1.0))
    m.set_ops(1, [])

    plan = _oracle_plan(ivs, cfg)
    st = oracle.GateState()
    ca, cb = ref.new_cache(), ref.new_cache()
    lg_ref, fr_ref, _ = ref.forward([dict(cache=ca, tokens=prompt, plan=plan, gate=st, frames=True),
                                     dict(cache=cb, tokens=other, frames=True)], act_scale=scale)
    out = m.forward([GpuSeq(0, 0, prompt), GpuSeq(1, 0, other)], capture=True)
    assert np.abs(out.logits - lg_ref).max() < LOGIT_TOL
    assert [int(x) for x in out.next_tokens] == [oracle.greedy(lg_ref[0]), oracle.greedy(lg_ref[1])]
    frames_ref = np.concatenate([fr_ref[0], fr_ref[1]])
    assert np.abs(out.frames.astype(np.int32) - frames_ref.astype(np.int32)).max() <= 1

    ref_open = [st.open(g) for g in range(5)]
    assert ref_open == [True, True, True, True, False]
    op, sc = m.gate_state(0)
    assert list(op) == ref_open
    ref_sc = np.array([st.score(g) for g in range(5)], np.float32)
    assert np.allclose(sc, ref_sc, rtol=1e-3, atol=1e-4)
    # the set op of the deciding layer starts exactly at the trigger row
    col = out.frames[:len(prompt), 5 * n + 3]
    q = oracle.compand(2.5 / SCALE)
    assert np.all(col[t:] == q) and not np.any(col[:t] == q)
    # the never-opening gate's set op (layer 4, value 9) left every row alone
    assert not np.any(out.frames[:len(prompt), 4 * n + 1] == oracle.compand(9.0 / SCALE))

    # later calls: every gate latched open applies from the first row, the layer-1 op included
    pos = len(prompt)
    tok = int(out.next_tokens[0])
    for step in range(6):
        lg_ref, fr_ref, _ = ref.forward([dict(cache=ca, tokens=np.array([tok], np.uint32), plan=plan, gate=st,
                                              frames=True)], act_scale=scale)
        o = m.forward([GpuSeq(0, pos, np.array([tok], np.uint32))], capture=True)
        assert np.abs(o.logits[0] - lg_ref[0]).max() < LOGIT_TOL, step
        assert int(o.next_tokens[0]) == oracle.greedy(lg_ref[0]), step
        assert np.abs(o.frames.astype(np.int32) - fr_ref[0].astype(np.int32)).max() <= 1
        _, sc = m.gate_state(0)
        assert np.allclose(sc, [st.score(g) for g in range(5)], rtol=1e-3, atol=1e-4), step
        assert o.frames[0, 5 * n + 3] == q
        pos += 1
        tok = int(o.next_tokens[0])

    # a fresh gate state closes every gate until a detector fires again
    m.reset_gates(0)
    op, sc = m.gate_state(0)
    assert not op.any() and not sc.any()
    st = oracle.GateState()
    lg_ref, _, _ = ref.forward([dict(cache=ca, tokens=np.array([tok], np.uint32), plan=plan, gate=st)])
    o = m.forward([GpuSeq(0, pos, np.array([tok], np.uint32))])
    assert np.abs(o.logits[0] - lg_ref[0]).max() < LOGIT_TOL
    assert list(m.gate_state(0)[0]) == [st.open(g) for g in range(5)]
    m.close()


@pytest.mark.gpu
def test_gated_decode_loop_matches_step_calls(gate_ckpt, gate_ref, cuda):
    """evie_decode_greedy with a gated plan (the detector kernel inside the captured step graph) gives the tokens and
    gate states of per-step evie_forward calls."""
    from evie_b200.gpu import GpuSeq

    cfg = gate_ref.cfg
    L, n = cfg.n_layers, cfg.intermediate
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, 2048, k).astype(np.uint32) for k in (23, 9)]
    # a low threshold on one detector, so that the gate may open at any step
    ivs = [Intervention(2, 7, 1.5, "add", gate=Gate([Detector(4, 33, 1.0)], 0.02)),
           Intervention(6, 50, 0.0, "mul", gate=Gate([Detector(4, 33, 1.0), Detector(6, 8, 2.0)], 0.05))]
    plan = Plan.compile(ivs, L, n, lambda l, nn: 1.0)
    results = []
    for mode in ("loop", "calls"):
        m = _gpu(gate_ckpt, max_ctx=128, slots=2, max_rows=64)
        m.set_plan(0, plan)
        m.set_plan(1, plan)
        out = m.forward([GpuSeq(i, 0, p) for i, p in enumerate(prompts)], want_logits=False)
        m.reset_gates(0)  # slot 0 starts the decode closed, slot 1 keeps what its prompt opened
        first = out.next_tokens.copy()
        seqs = [GpuSeq(i, len(p), first[i:i + 1]) for i, p in enumerate(prompts)]
        if mode == "loop":
            toks = m.decode_greedy(seqs, 8)
        else:
            toks, cur = [], first.copy()
            for step in range(8):
                o = m.forward([GpuSeq(i, len(p) + step, cur[i:i + 1]) for i, p in enumerate(prompts)],
                              want_logits=False)
                cur = o.next_tokens.copy()
                toks.append(cur)
            toks = np.stack(toks)
        results.append((toks, m.gate_state(0), m.gate_state(1)))
        m.close()
    assert np.array_equal(results[0][0], results[1][0])
    for k in (1, 2):
        assert np.array_equal(results[0][k][0], results[1][k][0])
        assert np.array_equal(results[0][k][1], results[1][k][1])


@pytest.mark.gpu
def test_plan_limits_are_reported(gate_ckpt, cuda):
    from evie_b200 import EvieError

    m = _gpu(gate_ckpt, max_ctx=64, slots=1, max_rows=16)
    bad_gate = Plan(ops=[(1, 2, 1, 0.5, 3)], thresholds=[0.0])
    with pytest.raises(EvieError, match="gate"):
        m.set_plan(0, bad_gate)
    too_many = Plan(ops=[], thresholds=[0.0] * 33)
    with pytest.raises(EvieError, match="gates"):
        m.set_plan(0, too_many)
    bad_det = Plan(ops=[(1, 2, 1, 0.5, 0)], thresholds=[0.0], detectors=[(1, 0, 0, 1.0)])
    with pytest.raises(EvieError, match="detector"):
        m.set_plan(0, bad_det)
    m.close()


def test_plan_compile_follows_reference_rules():
    """steering.rs:118-139 on the host: disabled and out-of-range interventions dropped, f32 dose x unit for Add,
    a gate index only for gates with detectors, out-of-range detectors dropped, last layer = deepest kept one."""
    ivs = [
        Intervention(0, 1, 0.7, "add"),
        Intervention(1, 2, 5.0, "mul", enabled=False),
        Intervention(9, 0, 1.0, "add"),                                      # layer out of range
        Intervention(2, 3, -1.0, "set", gate=Gate([], 1.0)),                 # empty gate: ungated
        Intervention(3, 4, 2.0, "add", gate=Gate([Detector(2, 5), Detector(7, 1, 0.5), Detector(3, 99)], 0.25)),
        Intervention(1, 1, 1.0, "mul", gate=Gate([Detector(8, 0)], -2.0)),   # no detector in range
    ]
    p = Plan.compile(ivs, 8, 64, lambda l, n: 0.1 * (l + 1))
    assert [o[:3] for o in p.ops] == [(0, 1, 1), (2, 3, 3), (3, 4, 1), (1, 1, 2)]
    assert p.ops[0][3] == float(np.float32(0.7) * np.float32(0.1))
    assert p.ops[2][3] == float(np.float32(2.0) * np.float32(np.float32(0.1 * 4)))
    assert [o[4] for o in p.ops] == [-1, -1, 0, 1]
    assert p.thresholds == [0.25, -2.0]
    assert p.detectors == [(0, 2, 5, 1.0), (0, 7, 1, 0.5)]
    assert p.last_layer == [7, 0]
