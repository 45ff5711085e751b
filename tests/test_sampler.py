"""The device sampler (evie_sample, evie_set_sampler) against the oracle's restatement of evie-core's Sampler
(crates/evie-core/src/sampling.rs:21-93).

Bar: the same tokens and the same generator states, on the same f32 logits. The oracle is pinned to splitmix64's
published output sequence (state 0: 0xe220a8397b1dcdaf, 0x6e789e6aa1b965f4, 0x06c45d188009454f) and to a second,
pure-Python restatement of Sampler::sample on small vocabularies."""
import math

import numpy as np
import pytest

import oracle

M64 = (1 << 64) - 1
GOLDEN = 0x9E3779B97F4A7C15


def _state(seed: int) -> int:
    return ((seed * GOLDEN) & M64) ^ 0xD1B54A32D192ED03


def _seed_for_state(state: int) -> int:
    """The seed whose Sampler::new state is `state` (the multiplier is odd, so invertible mod 2^64)."""
    return ((state ^ 0xD1B54A32D192ED03) * pow(GOLDEN, -1, 1 << 64)) & M64


def test_splitmix64_known_answers():
    """Sampler::uniform from state 0: the first three splitmix64 outputs' top 24 bits are 0.883, 0.431, 0.026; on
    two equal logits at temperature 1 a draw u picks token 0 iff u <= 0.5."""
    s = oracle.Sampler(1.0, 1.0, 0.0, 1.0, _seed_for_state(0))
    assert s.rng == 0
    assert [s.sample(np.zeros(2, np.float32), []) for _ in range(3)] == [1, 0, 0]
    assert s.rng == (3 * GOLDEN) & M64
    for z, u in ((0xE220A8397B1DCDAF, 0xE220A8), (0x6E789E6AA1B965F4, 0x6E789E), (0x06C45D188009454F, 0x06C45D)):
        assert z >> 40 == u


def test_library_seed_state():
    from evie_b200 import lib

    for seed in (0, 1, 42, 2**63 + 5, M64):
        assert lib().evie_sampler_seed_state(seed) == _state(seed)


def _py_sample(logits, hist, T, top_p, min_p, rep, state):
    """Sampler::sample restated in Python with numpy f32 scalars (small vocabularies only)."""
    f = np.float32
    lg = np.array(logits, np.float32)
    if rep != 1.0 and len(hist):
        for t in sorted(set(int(x) for x in hist)):
            if t < lg.size:
                lg[t] = lg[t] / f(rep) if lg[t] > 0 else lg[t] * f(rep)
    order = sorted(range(lg.size), key=lambda i: (-float(lg[i]), i))
    if T <= 0:
        return order[0], state
    cand = order[:512]
    top = lg[cand[0]]
    probs = [(i, f(math.exp(float((lg[i] - top) / f(T))))) for i in cand]
    total = f(0)
    for _, p in probs:
        total = f(total + p)
    probs = [(i, f(p / total)) for i, p in probs]
    if min_p > 0:
        floor = f(probs[0][1] * f(min_p))
        probs = [x for x in probs if x[1] >= floor]
    if top_p < 1:
        acc, keep = f(0), 0
        for _, p in probs:
            acc = f(acc + p)
            keep += 1
            if acc >= f(top_p):
                break
        probs = probs[:max(keep, 1)]
    total = f(0)
    for _, p in probs:
        total = f(total + p)
    state = (state + GOLDEN) & M64
    z = state
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    z ^= z >> 31
    r = f(f(z >> 40) / f(1 << 24)) * total
    for i, p in probs:
        r = f(r - p)
        if r <= 0:
            return i, state
    return (probs[-1][0] if probs else cand[0]), state


PARAMS = [
    dict(temperature=0.0, top_p=1.0, min_p=0.0, repetition_penalty=1.0),
    dict(temperature=0.0, top_p=1.0, min_p=0.0, repetition_penalty=1.3),
    dict(temperature=0.7, top_p=1.0, min_p=0.0, repetition_penalty=1.0),
    dict(temperature=1.3, top_p=0.9, min_p=0.0, repetition_penalty=1.2),
    dict(temperature=0.9, top_p=0.5, min_p=0.05, repetition_penalty=0.8),
    dict(temperature=1.0, top_p=1.0, min_p=1.5, repetition_penalty=1.0),  # min-p above 1 keeps nothing
]


def _oracle_sampler(p, seed):
    return oracle.Sampler(p["temperature"], p["top_p"], p["min_p"], p["repetition_penalty"], seed)


def test_oracle_matches_python_restatement():
    rng = np.random.default_rng(3)
    for V in (7, 300, 700):
        for k, p in enumerate(PARAMS):
            s = _oracle_sampler(p, 100 + k)
            state = s.rng
            for step in range(6):
                lg = (rng.normal(size=V) * 2).astype(np.float32)
                if step % 2:
                    lg = np.round(lg * 2) / 2  # ties
                hist = rng.integers(0, V + 5, rng.integers(0, 40))
                want, state = _py_sample(lg, hist, p["temperature"], p["top_p"], p["min_p"],
                                         p["repetition_penalty"], state)
                assert s.sample(lg, hist) == want, (V, k, step)
                assert s.rng == state


@pytest.mark.gpu
@pytest.mark.parametrize("V", [248320, 300])
def test_sample_op_matches_oracle(V, cuda):
    import torch

    from evie_b200 import ops

    rng = np.random.default_rng(5 + V)
    B = len(PARAMS) * 2
    params = PARAMS + PARAMS
    seeds = list(range(11, 11 + B))
    refs = [_oracle_sampler(p, sd) for p, sd in zip(params, seeds)]
    states = [ops.sampler_seed_state(sd) for sd in seeds]
    assert states == [r.rng for r in refs]
    for rnd in range(12):
        lg = (rng.normal(size=(B, V)) * 3).astype(np.float32)
        if rnd % 3 == 1:
            lg[B // 2:] = np.round(lg[B // 2:])  # wide ties across the 512-candidate cut
        if rnd % 3 == 2:
            lg[:, ::7] = 0.0
            lg[:, 1::7] = -0.0
        hists = [rng.integers(0, V + 10, rng.integers(0, 400)).astype(np.uint32) for _ in range(B)]
        got = ops.sample(torch.from_numpy(lg).to(cuda), params, states, hists)
        want = [r.sample(lg[b], hists[b]) for b, r in enumerate(refs)]
        assert list(got) == want, rnd
        assert states == [r.rng for r in refs], rnd


@pytest.fixture(scope="module")
def samp_ckpt(tmp_path_factory):
    from evie_b200 import checkpoint as ck

    path = str(tmp_path_factory.mktemp("sckpt") / "tiny")
    ck.write_checkpoint(path, ck.tiny_config(vocab_size=2048, num_hidden_layers=4), seed=2)
    return path


@pytest.mark.gpu
def test_model_sampler_matches_oracle_on_device_logits(samp_ckpt, cuda):
    """Per-slot samplers inside evie_forward: every sampled token equals the oracle Sampler's pick from the same
    logits with the worker's history (prompt ids + generated tokens, worker.rs:241, 320); a greedy slot in the same
    batch keeps the argmax."""
    from evie_b200.gpu import GpuModel, GpuSeq

    m = GpuModel(samp_ckpt, max_ctx=128, slots=2, max_rows=64)
    p = dict(temperature=0.8, top_p=0.9, min_p=0.02, repetition_penalty=1.2)
    m.set_sampler(0, seed=3, **p)
    ref = _oracle_sampler(p, 3)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, 2048, 19).astype(np.uint32), rng.integers(0, 2048, 7).astype(np.uint32)]
    out = m.forward([GpuSeq(i, 0, q) for i, q in enumerate(prompts)])
    hist = list(prompts[0])
    assert int(out.next_tokens[0]) == ref.sample(out.logits[0], hist)
    assert int(out.next_tokens[1]) == oracle.greedy(out.logits[1])
    pos = [len(q) for q in prompts]
    toks = [int(out.next_tokens[0]), int(out.next_tokens[1])]
    for step in range(10):
        hist.append(toks[0])
        out = m.forward([GpuSeq(i, pos[i], np.array([toks[i]], np.uint32)) for i in range(2)])
        assert int(out.next_tokens[0]) == ref.sample(out.logits[0], hist), step
        assert int(out.next_tokens[1]) == oracle.greedy(out.logits[1]), step
        pos = [x + 1 for x in pos]
        toks = [int(out.next_tokens[0]), int(out.next_tokens[1])]
    # back to greedy: plain argmax again
    m.set_sampler(0)
    out = m.forward([GpuSeq(0, pos[0], np.array([toks[0]], np.uint32))])
    assert int(out.next_tokens[0]) == oracle.greedy(out.logits[0])
    m.close()


@pytest.mark.gpu
def test_sampled_decode_loop_matches_step_calls(samp_ckpt, cuda):
    """evie_decode_greedy with stochastic samplers (the sampler inside the captured step graph) draws the same
    tokens as per-step evie_forward calls: the generator states live on the device."""
    from evie_b200.gpu import GpuModel, GpuSeq

    rng = np.random.default_rng(12)
    prompts = [rng.integers(0, 2048, n).astype(np.uint32) for n in (11, 25, 4)]
    results = []
    for mode in ("loop", "calls"):
        m = GpuModel(samp_ckpt, max_ctx=128, slots=3, max_rows=64)
        m.set_sampler(0, temperature=1.0, top_p=0.95, seed=7)
        m.set_sampler(2, temperature=0.6, repetition_penalty=1.5, seed=9)
        out = m.forward([GpuSeq(i, 0, p) for i, p in enumerate(prompts)], want_logits=False)
        first = out.next_tokens.copy()
        if mode == "loop":
            toks = m.decode_greedy([GpuSeq(i, len(p), first[i:i + 1]) for i, p in enumerate(prompts)], 12)
        else:
            toks, cur = [], first.copy()
            for step in range(12):
                o = m.forward([GpuSeq(i, len(p) + step, cur[i:i + 1]) for i, p in enumerate(prompts)],
                              want_logits=False)
                cur = o.next_tokens.copy()
                toks.append(cur)
            toks = np.stack(toks)
        results.append((first, toks))
        m.close()
    assert np.array_equal(results[0][0], results[1][0])
    assert np.array_equal(results[0][1], results[1][1])
