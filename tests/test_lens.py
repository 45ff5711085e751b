"""Lenses and readouts (crates/evie-core/src/lens.rs, analysis.rs): the oracle's restatement against float64 numpy,
the host logic (lens files, top-k, the ranking of search hits) against plain restatements of the reference's
loops, and the device calls (evie_set_lens, evie_lens_logits, evie_neuron_logits, evie_neuron_sigma through a
lens, evie_search_scores) against the oracle.

The lens is a random f16 (or bf16) map per layer, I + 0.05 N(0, 1), on layers 0 and 2 of a 4-layer model with
target layer 2: layer 1 has no map and layer 3 lies past the target, so both read out with the identity."""
import numpy as np
import pytest

import oracle
from evie_b200 import checkpoint as ck
from evie_b200 import lens as lz

PRE = "model.language_model."


@pytest.fixture(scope="module")
def lens_ckpt(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("lens") / "tiny")
    ck.write_checkpoint(path, ck.tiny_config(vocab_size=2048, num_hidden_layers=4), seed=4)
    return path


def _maps(d, kind, seed=9):
    rng = np.random.default_rng(seed)
    out = {}
    for l in (0, 2):
        m = (np.eye(d) + 0.05 * rng.standard_normal((d, d))).astype(np.float32)
        if kind == "f16":
            out[l] = m.astype(np.float16).view(np.uint16)
        else:
            out[l] = (m.view(np.uint32) >> 16).astype(np.uint16)  # bf16 by truncation: any bf16 values will do
    return out


def _widen(bits, kind):
    if kind == "f16":
        return bits.view(np.float16).astype(np.float64)
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def _weights(path):
    W = ck.read_tensor(path, PRE + "embed_tokens.weight").astype(np.float64)  # tied LM head [V][d]
    g = 1.0 + ck.read_tensor(path, PRE + "norm.weight").astype(np.float64)
    return W, g


def _np_unembed(x, W, g, eps):
    ms = (x * x).mean(axis=1, keepdims=True)
    return (x / np.sqrt(ms + eps) * g) @ W.T


def _np_map(lens, l, target=2):
    return None if l > target or l not in lens else lens[l]


def _close(a, b, rel):
    scale = float(np.abs(b).max())
    return float(np.abs(a - b).max()) <= rel * scale + 1e-6


@pytest.fixture(scope="module")
def ref(lens_ckpt):
    m = oracle.Model(lens_ckpt)
    yield m


# ---------------------------------------------------------------------------------------------- CPU: the oracle

@pytest.mark.parametrize("kind", ["f16", "bf16"])
def test_oracle_lens_logits_match_numpy(lens_ckpt, ref, kind):
    cfg = ref.cfg
    d = cfg.hidden
    maps = _maps(d, kind)
    ref.set_lens(maps, kind, 2)
    try:
        W, g = _weights(lens_ckpt)
        J = {l: _widen(m, kind).reshape(d, d) for l, m in maps.items()}
        x = np.random.default_rng(1).standard_normal((5, d)).astype(np.float32)
        for layer in range(cfg.n_layers):
            got = ref.lens_logits(layer, x)
            j = _np_map(J, layer)
            t = x.astype(np.float64) if j is None else x.astype(np.float64) @ j.T
            assert _close(got, _np_unembed(t, W, g, cfg.eps), 1e-5), layer
        # identity layers give the plain logit lens exactly
        ref.clear_lens()
        plain = ref.lens_logits(3, x)
        ref.set_lens(maps, kind, 2)
        assert np.array_equal(ref.lens_logits(3, x), plain)
        assert np.array_equal(ref.lens_logits(1, x), plain)
    finally:
        ref.clear_lens()


def test_oracle_neuron_logits_and_sigma_match_numpy(lens_ckpt, ref):
    cfg = ref.cfg
    d, n = cfg.hidden, cfg.intermediate
    maps = _maps(d, "f16")
    J = {l: _widen(m, "f16").reshape(d, d) for l, m in maps.items()}
    ref.set_lens(maps, "f16", 2)
    try:
        W, g = _weights(lens_ckpt)
        neurons = [(2, 5), (0, 17), (3, 255), (2, 0), (1, 100)]
        got = ref.neuron_logits(neurons)
        rows = []
        for l, i in neurons:
            w = ck.read_tensor(lens_ckpt, PRE + f"layers.{l}.mlp.down_proj.weight").astype(np.float64)[:, i]
            j = _np_map(J, l)
            rows.append(w if j is None else j @ w)
        assert _close(got, _np_unembed(np.stack(rows), W, g, cfg.eps), 1e-5)
        # neuron_sigma through the lens: sigma_n = sqrt(u^T M u), u = J_l w_n (analysis.rs:183-201)
        sig, mean, ms = ref.neuron_sigma()
        V = W.shape[0]
        s = min(16384, V)
        x = ((W[:: V // s][:s] - mean) * g).astype(np.float32)
        xw = (x * np.float32(64.0)).astype(np.float16).astype(np.float64)
        cov = (x.astype(np.float64).T @ xw).astype(np.float32) * np.float32(1.0 / (s * 64.0))
        M = (cov / np.float32(ms)).astype(np.float16).astype(np.float64)
        for l in range(cfg.n_layers):
            D = ck.read_tensor(lens_ckpt, PRE + f"layers.{l}.mlp.down_proj.weight").astype(np.float64)  # [d][n]
            j = _np_map(J, l)
            U = D if j is None else j @ D
            want = np.sqrt(np.maximum((U * (M @ U)).sum(0) * ms, 1e-30))
            assert np.allclose(sig[l * n:(l + 1) * n], want, rtol=2e-3, atol=0), l
    finally:
        ref.clear_lens()


def _search_reference_order(z_up, z_dn, limit):
    """analysis.rs:222-250 as written there: per layer a list of hits in neuron order (+ then -), stable sort by z
    descending, truncate; concatenate; stable sort; truncate."""
    L, n = z_up.shape
    allh = []
    for l in range(L):
        best = []
        for i in range(n):
            best.append((l, i, 1, float(z_up[l, i])))
            best.append((l, i, -1, float(z_dn[l, i])))
        best.sort(key=lambda h: -h[3])
        allh.extend(best[:limit])
    allh.sort(key=lambda h: -h[3])
    return allh[:limit]


def test_rank_hits_follows_the_reference_order():
    rng = np.random.default_rng(3)
    z_up = rng.integers(-3, 4, (3, 40)).astype(np.float32)  # many exact ties
    z_dn = rng.integers(-3, 4, (3, 40)).astype(np.float32)
    for limit in (1, 7, 50, 500):
        got = [(h.layer, h.neuron, h.sign, h.z) for h in lz.rank_hits(z_up, z_dn, limit)]
        assert got == _search_reference_order(z_up, z_dn, limit)


def test_oracle_search_matches_the_ranking_of_numpy_scores(lens_ckpt, ref):
    """The oracle's search against rank_hits over float64 scores; near-ties may order differently, so the hit
    z values are compared and the hits compared where the z gap exceeds f32 noise."""
    cfg = ref.cfg
    d, n = cfg.hidden, cfg.intermediate
    maps = _maps(d, "f16")
    J = {l: _widen(m, "f16").reshape(d, d) for l, m in maps.items()}
    ref.set_lens(maps, "f16", 2)
    try:
        sig, mean, _ = ref.neuron_sigma()
        W, g = _weights(lens_ckpt)
        toks = [3, 1999, 640]
        a = (W[toks] - mean.astype(np.float64)) * g
        z_up = np.zeros((cfg.n_layers, n), np.float32)
        z_dn = np.zeros((cfg.n_layers, n), np.float32)
        for l in range(cfg.n_layers):
            D = ck.read_tensor(lens_ckpt, PRE + f"layers.{l}.mlp.down_proj.weight").astype(np.float64)
            j = _np_map(J, l)
            pulled = a if j is None else a @ j
            z = (pulled @ D) / sig[l * n:(l + 1) * n]
            z_up[l], z_dn[l] = z.max(0), (-z).max(0)
        want = lz.rank_hits(z_up, z_dn, 25)
        got = ref.search(toks, mean, sig, 25)
        assert len(got) == 25
        assert np.allclose([h[3] for h in got], [h.z for h in want], rtol=1e-4, atol=1e-5)
        zs = [h.z for h in want]
        for i, h in enumerate(want):
            gap = min(abs(zs[i] - zs[i - 1]) if i else 1.0, abs(zs[i] - zs[i + 1]) if i + 1 < len(zs) else 1.0)
            if gap > 1e-3 * max(1.0, abs(h.z)):
                assert got[i][:3] == (h.layer, h.neuron, h.sign), i
    finally:
        ref.clear_lens()


def test_topk_ties_follow_kernels_rs():
    v = np.array([1.0, 3.0, 3.0, -2.0, 3.0, 0.5, 1.0], np.float32)
    for k in range(0, 9):
        idx, val = oracle.topk(v, k)
        assert lz.topk(v, k) == [(int(i), float(x)) for i, x in zip(idx, val)]


def test_lens_file_loading(tmp_path):
    import torch

    d, L = 8, 4
    mk = lambda dt: torch.eye(d, dtype=dt) + 0.5  # noqa: E731
    p = str(tmp_path / "l.pt")
    torch.save({"J": {0: mk(torch.float16), 2: mk(torch.float16), 3: "not a tensor"}, "n_prompts": 12,
                "provenance": {"target_layer": 2, "method": "jacobian++"}}, p)
    lens = lz.Lens.load(p, "j", L, d)
    assert (lens.target_layer, lens.kind, lens.n_prompts, lens.method) == (2, "f16", 12, "jacobian++")
    assert sorted(lens.maps) == [0, 2]
    assert np.array_equal(lens.maps[2].view(np.float16), mk(torch.float16).numpy())
    assert lens.map(3) is None and lens.map(1) is None and lens.map(2) is not None
    # default target layer: one past the highest mapped layer, capped at the last layer
    torch.save({"J": {1: mk(torch.bfloat16)}}, p)
    lens = lz.Lens.load(p, "j", L, d)
    assert (lens.target_layer, lens.kind, lens.method) == (2, "bf16", "jacobian")
    torch.save({"J": {3: mk(torch.bfloat16)}}, p)
    assert lz.Lens.load(p, "j", L, d).target_layer == 3
    for bad, msg in [({"X": {}}, "no `J`"), ({"J": {4: mk(torch.float16)}}, "out of range"),
                     ({"J": {0: torch.eye(d + 1, dtype=torch.float16)}}, "shape"),
                     ({"J": {0: torch.eye(d)}}, "dtype"),
                     ({"J": {0: mk(torch.float16), 1: mk(torch.bfloat16)}}, "mix")]:
        torch.save(bad, p)
        with pytest.raises(ValueError, match=msg):
            lz.Lens.load(p, "j", L, d)


# ---------------------------------------------------------------------------------------------- GPU: the device

def _gpu(path):
    from evie_b200.gpu import GpuModel

    return GpuModel(path, max_ctx=64, slots=1, max_rows=16)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["f16", "bf16"])
def test_device_lens_logits_and_sigma(lens_ckpt, ref, kind, cuda):
    cfg = ref.cfg
    d = cfg.hidden
    maps = _maps(d, kind)
    x = np.random.default_rng(2).standard_normal((70, d)).astype(np.float32)  # two unembedding blocks
    ref.set_lens(maps, kind, 2)
    m = _gpu(lens_ckpt)
    try:
        m.set_lens(lz.Lens("t", 2, maps, kind))
        for layer in range(cfg.n_layers):
            assert _close(m.lens_logits(layer, x), ref.lens_logits(layer, x), 2e-5), layer
        sig, mean, ms = m.neuron_sigma()
        sig_r, mean_r, ms_r = ref.neuron_sigma()
        assert np.array_equal(mean, mean_r)
        assert abs(ms - ms_r) <= 1e-5 * ms_r
        assert np.allclose(sig, sig_r, rtol=1e-3, atol=0)
        m.set_lens(None)
        ref.clear_lens()
        assert _close(m.lens_logits(2, x[:3]), ref.lens_logits(2, x[:3]), 2e-5)
    finally:
        m.close()
        ref.clear_lens()


@pytest.mark.gpu
def test_device_neuron_logits_readouts_and_search(lens_ckpt, ref, cuda):
    cfg = ref.cfg
    d = cfg.hidden
    maps = _maps(d, "f16")
    ref.set_lens(maps, "f16", 2)
    m = _gpu(lens_ckpt)
    try:
        m.set_lens(lz.Lens("t", 2, maps, "f16"))
        rng = np.random.default_rng(5)
        neurons = [(int(l), int(i))
                   for l, i in zip(rng.integers(0, cfg.n_layers, 60), rng.integers(0, cfg.intermediate, 60))]
        got, want = m.neuron_logits(neurons), ref.neuron_logits(neurons)
        assert _close(got, want, 2e-5)
        # readouts: each device top-k token is within f32 noise of the oracle's k-th best logit
        for r, row in zip(lz.neuron_readouts(m, neurons[:10], 8), want[:10]):
            kth = np.sort(row)[-8]
            assert all(row[t] >= kth - 1e-4 * np.abs(row).max() for t, _ in r.up)
            kth_dn = np.sort(row)[7]
            assert all(row[t] <= kth_dn + 1e-4 * np.abs(row).max() for t, _ in r.down)
        sig, mean, _ = ref.neuron_sigma()
        toks = [3, 1999, 640]
        hits = lz.search(m, toks, mean, sig, 25)
        hits_ref = ref.search(toks, mean, sig, 25)
        assert np.allclose([h.z for h in hits], [h[3] for h in hits_ref], rtol=1e-4, atol=1e-5)
        zs = [h[3] for h in hits_ref]
        for i, h in enumerate(hits_ref):
            gap = min(abs(zs[i] - zs[i - 1]) if i else 1.0, abs(zs[i] - zs[i + 1]) if i + 1 < len(zs) else 1.0)
            if gap > 1e-3 * max(1.0, abs(h[3])):
                assert (hits[i].layer, hits[i].neuron, hits[i].sign) == h[:3], i
    finally:
        m.close()
        ref.clear_lens()


def test_lens_calls_check_their_arguments(lens_ckpt):
    """Argument checks run before any device work (no GPU needed)."""
    from evie_b200 import lib

    L = lib()
    assert L.evie_set_lens(None, None, 0, 0, 0) == 1
    assert L.evie_lens_logits(None, 0, None, 0, None) == 1
    assert L.evie_neuron_logits(None, None, None, 0, None) == 1
    assert L.evie_search_scores(None, None, 0, None, None, None, None) == 1
    assert L.evie_clear_lens(None) == 1
    assert b"null context" in L.evie_last_global_error()
