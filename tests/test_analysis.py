"""Offline analysis (evie_neuron_sigma): evie-core's UnembedStats::compute and neuron_sigma without a lens
(crates/evie-core/src/analysis.rs:129-201) on the device, against the oracle's restatement, which is itself checked
against an independent float64 numpy formulation of the same formulas (same f16 roundings)."""
import numpy as np
import pytest

import oracle
from evie_b200 import checkpoint as ck


@pytest.fixture(scope="module")
def an_ckpt(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("an") / "tiny")
    ck.write_checkpoint(path, ck.tiny_config(vocab_size=2048, num_hidden_layers=4), seed=3)
    return path


def _numpy_sigma(path, cfg):
    """analysis.rs:129-201 in float64 numpy, with the reference's f16 roundings of the two weight operands."""
    pre = "model.language_model."
    W = ck.read_tensor(path, pre + "embed_tokens.weight").astype(np.float32)  # tied LM head [V][d]
    g = (1.0 + ck.read_tensor(path, pre + "norm.weight").astype(np.float32)).astype(np.float32)
    V, d = W.shape
    mean = (W.astype(np.float64).sum(0) / V).astype(np.float32)
    s = min(16384, V)
    stride = V // s
    x = ((W[::stride][:s] - mean) * g).astype(np.float32)  # [s][d]
    xw = (x * np.float32(64.0)).astype(np.float16).astype(np.float64)
    cov = (x.astype(np.float64).T @ xw).astype(np.float32) * np.float32(1.0 / (s * 64.0))
    m_scale = max(float(np.abs(cov).max()), 1e-30)
    M = (cov / np.float32(m_scale)).astype(np.float16).astype(np.float64)
    sig = []
    for l in range(cfg.n_layers):
        D = ck.read_tensor(path, pre + f"layers.{l}.mlp.down_proj.weight").astype(np.float64)  # [d][n]
        mu = M @ D  # [d][n]
        sig.append(np.sqrt(np.maximum((D * mu).sum(0) * m_scale, 1e-30)))
    return np.concatenate(sig).astype(np.float32), mean, m_scale


def test_oracle_matches_numpy(an_ckpt):
    m = oracle.Model(an_ckpt)
    sig, mean, ms = m.neuron_sigma()
    sig_np, mean_np, ms_np = _numpy_sigma(an_ckpt, m.cfg)
    assert np.array_equal(mean, mean_np)
    assert abs(ms - ms_np) <= 1e-5 * ms_np
    assert np.allclose(sig, sig_np, rtol=2e-3, atol=0)


@pytest.mark.gpu
def test_neuron_sigma_matches_oracle(an_ckpt, cuda):
    from evie_b200.gpu import GpuModel

    m_ref = oracle.Model(an_ckpt)
    sig_ref, mean_ref, ms_ref = m_ref.neuron_sigma()
    g = GpuModel(an_ckpt, max_ctx=64, slots=1, max_rows=16)
    sig, mean, ms = g.neuron_sigma()
    g.close()
    assert np.array_equal(mean, mean_ref)
    assert abs(ms - ms_ref) <= 1e-5 * ms_ref
    assert np.allclose(sig, sig_ref, rtol=1e-3, atol=0)
