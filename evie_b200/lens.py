"""Lenses and readouts: the host side of the analysis calls (crates/evie-core/src/lens.rs, analysis.rs).

The device computes the products (evie_set_lens, evie_lens_logits, evie_neuron_logits, evie_neuron_sigma,
evie_search_scores through GpuModel); this module reads lens files the way Lens::load does and ranks the device's
outputs the way the readout functions do:

  Lens.load         lens.rs:20-54   torch file with a `J` dict {layer: [d][d] f16/bf16}, provenance.target_layer
                                    (default: one past the highest mapped layer, capped at the last layer), method,
                                    n_prompts
  topk              kernels.rs:642-662  largest first, equal values in index order
  neuron_readouts   analysis.rs:70-81   top-k tokens of both poles of each neuron's write direction
  token_ranks       analysis.rs:84-105  best rank of any query token in each pole (0 = top)
  resid_readouts    analysis.rs:108-120 top-k tokens of residual-stream vectors (layer, vector)
  search            analysis.rs:213-251 hits (layer, neuron, sign, z) ranked from the device's per-neuron best z
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

NEURON_CHUNK = 48  # analysis.rs:73, 87: readouts are computed 48 neurons at a time


@dataclass
class Lens:
    """lens.rs:10-16: per-layer maps (uint16 bits of f16 or bf16 [d][d] matrices) and where they read out."""
    name: str
    target_layer: int
    maps: dict = field(default_factory=dict)
    kind: str = "f16"
    n_prompts: int = 0
    method: str = "jacobian"

    @classmethod
    def load(cls, path: str, name: str, n_layers: int, d: int) -> "Lens":
        """lens.rs:20-54. All maps of one file must share a dtype (the device holds one format per lens)."""
        import torch

        obj = torch.load(path, map_location="cpu", weights_only=True)
        J = obj.get("J") if isinstance(obj, dict) else None
        if not isinstance(J, dict):
            raise ValueError(f"{path}: no `J` dict (not a lens file?)")
        maps, kinds, max_src = {}, set(), 0
        for k, v in J.items():
            if isinstance(k, bool) or not isinstance(k, (int, np.integer)):
                raise ValueError(f"{path}: non-integer layer key {k!r}")
            layer = int(k)
            if not torch.is_tensor(v):
                continue
            if layer >= n_layers:
                raise ValueError(f"{path}: layer {layer} out of range for a {n_layers}-layer model")
            if tuple(v.shape) != (d, d):
                raise ValueError(f"{path}: layer {layer} map has shape {list(v.shape)}, expected [{d}, {d}]")
            if v.dtype == torch.float16:
                kinds.add("f16")
            elif v.dtype == torch.bfloat16:
                kinds.add("bf16")
            else:
                raise ValueError(f"{path}: unsupported lens dtype {v.dtype}")
            maps[layer] = v.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
            max_src = max(max_src, layer)
        if len(kinds) > 1:
            raise ValueError(f"{path}: maps mix f16 and bf16")
        prov = obj.get("provenance")
        prov = prov if isinstance(prov, dict) else {}
        tl = prov.get("target_layer")
        target = int(tl) if isinstance(tl, (int, np.integer)) and not isinstance(tl, bool) else min(max_src + 1,
                                                                                                  n_layers - 1)
        method = prov.get("method", prov.get("config_json"))
        method = method if isinstance(method, str) else "jacobian"
        n_prompts = obj.get("n_prompts", 0)
        n_prompts = int(n_prompts) if isinstance(n_prompts, (int, np.integer)) else 0
        return cls(name, target, maps, kinds.pop() if kinds else "f16", n_prompts, method)

    def map(self, layer: int):
        """lens.rs:57-62: the layer's map, or None (identity) past the target layer or where the file has none."""
        return None if layer > self.target_layer else self.maps.get(layer)


def _total_key(x: np.ndarray) -> np.ndarray:
    """f32 values as int64 keys in IEEE total order (Rust's f32::total_cmp)."""
    i = np.ascontiguousarray(x, np.float32).view(np.int32).astype(np.int64)
    return np.where(i < 0, -(i & 0x7FFFFFFF) - 1, i)


def topk(values: np.ndarray, k: int):
    """kernels.rs:642-662: the k largest (index, value), largest first, equal values in index order."""
    v = np.asarray(values, np.float32)
    k = min(k, v.size)
    if k <= 0:
        return []
    idx = np.argsort(-v.astype(np.float64), kind="stable")[:k]
    return [(int(i), float(v[i])) for i in idx]


@dataclass
class Readout:
    """analysis.rs:20-25: tokens the + pole pushes up (logits descending), and those the - pole pushes up."""
    up: list
    down: list


def neuron_readouts(model, neurons, k: int):
    """analysis.rs:70-81 over model.neuron_logits (the device's lens + unembedding)."""
    out = []
    for c0 in range(0, len(neurons), NEURON_CHUNK):
        logits = model.neuron_logits(neurons[c0:c0 + NEURON_CHUNK])
        for row in logits:
            out.append(Readout(topk(row, k), [(t, -x) for t, x in topk(-row, k)]))
    return out


def token_ranks(model, neurons, tokens):
    """analysis.rs:84-105: (best rank in the + pole, best rank in the - pole) per neuron; 0 = top, and the largest
    64-bit value when no token is inside the vocabulary."""
    none = 2 ** 64 - 1
    out = []
    for c0 in range(0, len(neurons), NEURON_CHUNK):
        logits = model.neuron_logits(neurons[c0:c0 + NEURON_CHUNK])
        for row in logits:
            ok = [int(t) for t in tokens if int(t) < row.size]

            def best(sign):
                r = [int(np.count_nonzero(sign * row > sign * row[t])) for t in ok]
                return min(r) if r else none

            out.append((best(1.0), best(-1.0)))
    return out


def resid_readouts(model, resids, k: int):
    """analysis.rs:108-120: top-k tokens of each (layer, residual vector) through the lens and the unembedding."""
    return [topk(model.lens_logits(layer, np.asarray(vec, np.float32)[None])[0], k) for layer, vec in resids]


@dataclass(frozen=True)
class Hit:
    """analysis.rs:204-210"""
    layer: int
    neuron: int
    sign: int
    z: float


def rank_hits(z_up: np.ndarray, z_dn: np.ndarray, limit: int):
    """analysis.rs:222-250 from the per-neuron best z of both poles ([layers][neurons] each): per layer the hits
    (neuron order, + pole before - pole) sorted by z descending, stable, cut to `limit`; then all layers merged in
    layer order and sorted and cut the same way."""
    L, n = z_up.shape
    merged = []
    for l in range(L):
        z = np.stack([z_up[l], z_dn[l]], axis=1).reshape(-1)  # neuron-major: (+, -) per neuron
        order = np.argsort(-_total_key(z), kind="stable")[:limit]
        merged.extend(Hit(l, int(i // 2), 1 if i % 2 == 0 else -1, float(z[i])) for i in order)
    keys = _total_key(np.array([h.z for h in merged], np.float32))
    return [merged[i] for i in np.argsort(-keys, kind="stable")[:limit]]


def search(model, tokens, mean: np.ndarray, sigma: np.ndarray, limit: int):
    """analysis.rs:213-251 over model.search_scores (the device's pullbacks, scores and per-neuron maxima)."""
    if len(tokens) == 0:
        return []
    z_up, z_dn = model.search_scores(tokens, mean, sigma)
    return rank_hits(z_up, z_dn, limit)
