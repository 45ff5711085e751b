"""CPU oracle: ctypes wrapper over ``oracle/liboracle.so``.

TEST INFRASTRUCTURE ONLY. A C++ restatement of evie-core's CPU engine (the Rust original cannot be built
here). Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this module,
and only as the checker; the product library (``evie_b200``) never imports, links or calls it.

Loading follows the reference's own loader:
  * ``load_config``   restates crates/evie-core/src/config.rs:79-137 (text_config nesting, rope_parameters,
                      rotary_dim = round(head_dim * partial_rotary_factor), default rope_theta 1e7);
  * ``SafeTensors``   restates crates/evie-core/src/weights.rs:33-123 (BF16/F16/F32, [C,1,K] conv as 2-D);
  * ``Model``         restates crates/evie-core/src/model.rs:137-203 (prefix detection, tied lm_head);
  * ``compile_plan``  restates crates/evie-core/src/steering.rs:118-139 (Add value x dose unit, gates).
"""
from __future__ import annotations

import ctypes as C
import json
import math
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None


def build() -> None:
    """Compiles liboracle.so in place (make)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = C.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


class _Cfg(C.Structure):
    _fields_ = [
        ("hidden", C.c_int), ("intermediate", C.c_int), ("n_layers", C.c_int), ("vocab", C.c_int),
        ("eps", C.c_float), ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int),
        ("rotary_dim", C.c_int), ("rope_theta", C.c_double), ("conv_kernel", C.c_int),
        ("lin_k_heads", C.c_int), ("lin_v_heads", C.c_int), ("lin_k_dim", C.c_int), ("lin_v_dim", C.c_int),
    ]


class _Seq(C.Structure):
    _fields_ = [
        ("cache", C.c_void_p), ("tokens", C.c_void_p), ("n", C.c_long), ("plan", C.c_void_p),
        ("gate", C.c_void_p), ("frames", C.c_void_p), ("resid", C.c_void_p),
    ]


def _declare(L):
    P, I, LG, F = C.c_void_p, C.c_int, C.c_long, C.c_float
    sig = {
        "oracle_set_threads": (None, [I]),
        "oracle_threads": (I, []),
        "oracle_matmul": (None, [P, LG, LG, P, LG, P]),
        "oracle_topk": (I, [P, LG, I, P, P]),
        "oracle_softmax": (None, [P, LG]),
        "oracle_dot": (F, [P, P, LG]),
        "oracle_gdn_decode": (None, [I, I, I, I, P, P, P, P, P, P, P]),
        "oracle_gdn_prefill": (None, [I, I, I, I, I, P, P, P, P, P, P, P]),
        "oracle_gqa_decode": (None, [I, I, I, I, I, P, P, P, P, I, P, P, F, P]),
        "oracle_gqa_rows": (None, [I, I, I, I, I, P, P, P, P, I, P, P, P, F, P]),
        "oracle_model_new": (P, [P, P]),
        "oracle_model_free": (None, [P]),
        "oracle_model_kv_bf16": (None, [P, I, F]),
        "oracle_model_set": (I, [P, I, I, P, I, LG, LG]),
        "oracle_cache_new": (P, [P]),
        "oracle_cache_free": (None, [P]),
        "oracle_cache_seed": (None, [P, P, LG, C.c_uint64]),
        "oracle_cache_clone": (P, [P]),
        "oracle_cache_pos": (LG, [P]),
        "oracle_cache_read": (LG, [P, I, I, P, LG]),
        "oracle_plan_new": (P, [I]),
        "oracle_plan_free": (None, [P]),
        "oracle_plan_add_op": (None, [P, I, I, I, F, I]),
        "oracle_plan_add_gate": (I, [P, F, I]),
        "oracle_plan_add_detector": (None, [P, I, I, I, F]),
        "oracle_gate_state_new": (P, []),
        "oracle_gate_state_free": (None, [P]),
        "oracle_gate_state_open": (I, [P, I]),
        "oracle_top_active": (I, [P, LG, I, P]),
        "oracle_neuron_sigma": (F, [P, P, P]),
        "oracle_lens_set": (None, [P, P, I, I, LG]),
        "oracle_lens_clear": (None, [P]),
        "oracle_lens_logits": (None, [P, I, P, LG, P]),
        "oracle_neuron_logits": (None, [P, P, P, LG, P]),
        "oracle_search": (LG, [P, P, LG, P, P, LG, P, P, P, P]),
        "oracle_sampler_new": (P, [F, F, F, F, C.c_uint64]),
        "oracle_sampler_free": (None, [P]),
        "oracle_sampler_rng": (C.c_uint64, [P]),
        "oracle_sampler_sample": (C.c_uint32, [P, P, LG, P, LG]),
        "oracle_gate_state_score": (F, [P, I]),
        "oracle_gate_state_partial": (LG, [P, I, P, LG]),
        "oracle_plan_begin": (None, [P, P, LG]),
        "oracle_plan_apply": (None, [P, I, P, LG, LG, P]),
        "oracle_forward": (None, [P, P, I, P, P, I, P]),
        "oracle_compand": (C.c_int8, [F]),
        "oracle_f32_to_f16": (C.c_uint16, [F]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def threads() -> int:
    return lib().oracle_threads()


# ---------------------------------------------------------------------------------------------------
# kernels (kernels.rs)

def matmul(w_bf16: np.ndarray, x: np.ndarray) -> np.ndarray:
    """Y[t, r] = sum_k W[r, k] X[t, k] with evie-core's dispatch by n (kernels.rs:163-184)."""
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[0]
    y = np.zeros((n, w.shape[0]), np.float32)
    lib().oracle_matmul(_p(w), w.shape[0], w.shape[1], _p(x), n, _p(y))
    return y


def topk(v: np.ndarray, k: int):
    v = np.ascontiguousarray(v, dtype=np.float32)
    idx = np.zeros(max(k, 1), np.uint32)
    val = np.zeros(max(k, 1), np.float32)
    n = lib().oracle_topk(_p(v), v.size, k, _p(idx), _p(val))
    return idx[:n].copy(), val[:n].copy()


def greedy(logits: np.ndarray) -> int:
    """sampling.rs:60-62 with temperature 0: topk(logits, 1)."""
    return int(topk(logits, 1)[0][0])


class Sampler:
    """sampling.rs:21-93: Sampler::new(params) and Sampler::sample(logits, history)."""

    def __init__(self, temperature=0.0, top_p=1.0, min_p=0.0, repetition_penalty=1.0, seed=0):
        self._h = lib().oracle_sampler_new(temperature, top_p, min_p, repetition_penalty, seed)

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.oracle_sampler_free(self._h)
            self._h = None

    @property
    def rng(self) -> int:
        return int(lib().oracle_sampler_rng(self._h))

    def sample(self, logits: np.ndarray, history) -> int:
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        h = np.ascontiguousarray(history, dtype=np.uint32)
        return int(lib().oracle_sampler_sample(self._h, _p(lg), lg.size, _p(h) if h.size else None, h.size))


def top_active(frame: np.ndarray, k: int) -> np.ndarray:
    """mcp.rs:242-256: flat indices of the k largest |q| of one i8 frame, equal |q| by lower index."""
    f = np.ascontiguousarray(frame, dtype=np.int8)
    out = np.zeros(max(k, 1), np.int32)
    n = lib().oracle_top_active(_p(f), f.size, k, _p(out))
    return out[:n].copy()


def compand(v: float) -> int:
    return int(lib().oracle_compand(float(v)))


# ---------------------------------------------------------------------------------------------------
# isolated ops

def gdn_decode(S, q, k, v, g, beta):
    """One gated-delta-rule step over [B, H] heads (model.rs:374-376, 501-524). S updated in place.

    S: [B,H,dk,dv] f32; q,k: [B,H,dk] bf16 bits (uint16); v: [B,H,dv] bf16 bits; g, beta: [B,H] f32.
    Returns o [B,H,dv] f32.
    """
    B, H, dk, dv = S.shape
    o = np.zeros((B, H, dv), np.float32)
    args = [np.ascontiguousarray(a) for a in (q, k, v, g, beta)]
    lib().oracle_gdn_decode(B, H, dk, dv, _p(S), *[_p(a) for a in args], _p(o))
    return o


def gdn_prefill(S, q, k, v, g, beta):
    """Token-sequential gated delta rule (evie-core has no chunked form). q,k,v: [B,T,H,d]; g,beta: [B,T,H]."""
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    o = np.zeros((B, T, H, dv), np.float32)
    args = [np.ascontiguousarray(a) for a in (q, k, v, g, beta)]
    lib().oracle_gdn_prefill(B, T, H, dk, dv, _p(S), *[_p(a) for a in args], _p(o))
    return o


def gqa_rows(q, kpages, vpages, page_table, row_seq, row_pos, gate, scale):
    """model.rs:445-464 for prefill rows: q, gate f32 [R, Hq, hd]; pages bf16 bits [P, Hkv, page, hd]; page_table
    [n_seqs, max_pages]; row r attends to positions 0..row_pos[r] of sequence row_seq[r]. Returns [R, Hq, hd]."""
    q = np.ascontiguousarray(q, np.float32)
    gate = np.ascontiguousarray(gate, np.float32)
    kpages = np.ascontiguousarray(kpages, np.uint16)
    vpages = np.ascontiguousarray(vpages, np.uint16)
    pt = np.ascontiguousarray(page_table, np.int32)
    rs = np.ascontiguousarray(row_seq, np.int32)
    rp = np.ascontiguousarray(row_pos, np.int32)
    R, Hq, hd = q.shape
    _, Hkv, page, _ = kpages.shape
    out = np.zeros((R, Hq, hd), np.float32)
    lib().oracle_gqa_rows(R, Hq, Hkv, hd, page, _p(q), _p(kpages), _p(vpages), _p(pt), pt.shape[1], _p(rs), _p(rp),
                          _p(gate), scale, _p(out))
    return out


def gqa_decode(q, kpages, vpages, page_table, ctx, gate, scale):
    """Gated GQA decode attention core (model.rs:445-464) over pages [P, Hkv, page, hd]."""
    B, Hq, hd = q.shape
    _, Hkv, page, _ = kpages.shape
    out = np.zeros((B, Hq, hd), np.float32)
    pt = np.ascontiguousarray(page_table, dtype=np.int32)
    cx = np.ascontiguousarray(ctx, dtype=np.int32)
    arrs = [np.ascontiguousarray(a) for a in (q, kpages, vpages)]
    g = np.ascontiguousarray(gate)
    lib().oracle_gqa_decode(B, Hq, Hkv, hd, page, _p(arrs[0]), _p(arrs[1]), _p(arrs[2]), _p(pt), pt.shape[1],
                            _p(cx), _p(g), float(scale), _p(out))
    return out


# ---------------------------------------------------------------------------------------------------
# config / weights / model

@dataclass
class Config:
    hidden: int
    intermediate: int
    n_layers: int
    layer_kinds: list  # "linear" | "full"
    vocab: int
    eps: float
    tie_embeddings: bool
    n_heads: int
    n_kv_heads: int
    head_dim: int
    rotary_dim: int
    rope_theta: float
    conv_kernel: int
    lin_k_heads: int
    lin_v_heads: int
    lin_k_dim: int
    lin_v_dim: int
    eos_ids: list = field(default_factory=list)

    def conv_dim(self) -> int:
        return 2 * self.lin_k_heads * self.lin_k_dim + self.lin_v_heads * self.lin_v_dim


def load_config(path: str) -> Config:
    """config.rs:79-137."""
    with open(path) as f:
        root = json.load(f)
    t = root.get("text_config", root)
    if t.get("rope_parameters") is not None:
        rp = t["rope_parameters"]
        theta, partial = float(rp["rope_theta"]), float(rp.get("partial_rotary_factor", 1.0))
    else:
        theta = float(t.get("rope_theta") if t.get("rope_theta") is not None else 10_000_000.0)
        partial = float(t.get("partial_rotary_factor") if t.get("partial_rotary_factor") is not None else 1.0)
    kinds = []
    for lt in t["layer_types"]:
        if lt == "linear_attention":
            kinds.append("linear")
        elif lt == "full_attention":
            kinds.append("full")
        else:
            raise ValueError(f"unsupported layer type {lt!r}")
    if len(kinds) != t["num_hidden_layers"]:
        raise ValueError(f"layer_types has {len(kinds)} entries for {t['num_hidden_layers']} layers")
    tie = t.get("tie_word_embeddings")
    if tie is None:
        tie = root.get("tie_word_embeddings") if isinstance(root.get("tie_word_embeddings"), bool) else False
    eos = []
    for v in (t.get("eos_token_id"), root.get("eos_token_id")):
        if isinstance(v, int):
            eos.append(v)
        elif isinstance(v, list):
            eos.extend(x for x in v if isinstance(x, int))
    rot = math.floor(t["head_dim"] * partial + 0.5)  # f64::round (half away from zero) for positive values
    return Config(
        hidden=t["hidden_size"], intermediate=t["intermediate_size"], n_layers=t["num_hidden_layers"],
        layer_kinds=kinds, vocab=t["vocab_size"], eps=float(np.float32(t["rms_norm_eps"])), tie_embeddings=bool(tie),
        n_heads=t["num_attention_heads"], n_kv_heads=t["num_key_value_heads"], head_dim=t["head_dim"],
        rotary_dim=rot, rope_theta=theta, conv_kernel=t["linear_conv_kernel_dim"],
        lin_k_heads=t["linear_num_key_heads"], lin_v_heads=t["linear_num_value_heads"],
        lin_k_dim=t["linear_key_head_dim"], lin_v_dim=t["linear_value_head_dim"], eos_ids=sorted(set(eos)),
    )


class SafeTensors:
    """weights.rs:33-123: every *.safetensors in a directory, memory-mapped."""

    _DT = {"BF16": np.uint16, "F16": np.float16, "F32": np.float32}

    def __init__(self, d: str):
        paths = sorted(os.path.join(d, p) for p in os.listdir(d) if p.endswith(".safetensors"))
        if not paths:
            raise FileNotFoundError(f"no .safetensors files in {d}")
        self.entries = {}
        self._maps = []
        for path in paths:
            mm = np.memmap(path, dtype=np.uint8, mode="r")
            n = int.from_bytes(bytes(mm[:8]), "little")
            header = json.loads(bytes(mm[8:8 + n]))
            base = 8 + n
            for name, v in header.items():
                if name == "__metadata__" or v["dtype"] not in self._DT:
                    continue
                s, e = v["data_offsets"]
                self.entries[name] = (mm, v["dtype"], list(v["shape"]), base + s, base + e)
            self._maps.append(mm)

    def has(self, name: str) -> bool:
        return name in self.entries

    def raw(self, name: str) -> tuple:
        mm, dt, shape, s, e = self.entries[name]
        arr = np.frombuffer(mm, dtype=np.uint8, count=e - s, offset=s).view(self._DT[dt])
        return dt, shape, arr

    def mat16(self, name: str) -> np.ndarray:
        dt, shape, arr = self.raw(name)
        if dt != "BF16":
            raise ValueError(f"{name}: the oracle reads bf16 matrices only, got {dt}")
        if len(shape) == 3 and shape[1] == 1:
            shape = [shape[0], shape[2]]
        if len(shape) != 2:
            raise ValueError(f"{name}: expected 2-D, got {shape}")
        return arr.reshape(shape)

    def f32s(self, name: str) -> np.ndarray:
        dt, _, arr = self.raw(name)
        if dt == "BF16":
            return (arr.astype(np.uint32) << 16).view(np.float32)
        return arr.astype(np.float32)


_MATS = {
    "linear_attn.in_proj_qkv.weight": 10, "linear_attn.in_proj_z.weight": 11, "linear_attn.in_proj_b.weight": 12,
    "linear_attn.in_proj_a.weight": 13, "linear_attn.out_proj.weight": 14,
    "self_attn.q_proj.weight": 20, "self_attn.k_proj.weight": 21, "self_attn.v_proj.weight": 22,
    "self_attn.o_proj.weight": 23, "mlp.gate_proj.weight": 30, "mlp.up_proj.weight": 31, "mlp.down_proj.weight": 32,
}
_VECS = {
    "input_layernorm.weight": 40, "post_attention_layernorm.weight": 41, "self_attn.q_norm.weight": 43,
    "self_attn.k_norm.weight": 44, "linear_attn.conv1d.weight": 45, "linear_attn.A_log": 46,
    "linear_attn.dt_bias": 47, "linear_attn.norm.weight": 48,
}


class Model:
    """model.rs:137-203 over the oracle engine."""

    def __init__(self, ckpt_dir: str, kv_bf16: bool = False, kv_perturb: float = 0.0):
        """kv_bf16: round every appended key and value to bf16 (the GPU's paged-cache format), the oracle's one
        documented deviation from model.rs:441-442, which appends f32 rows. Off by default.
        kv_perturb (with kv_bf16): scale each key and value by 1 + kv_perturb * r, r uniform in [-1, 1) from a fixed
        generator, before rounding. A test aid that measures how far the bf16 rounding alone moves the logits when
        the values before rounding differ at the level of f32 reordering."""
        self.cfg = load_config(os.path.join(ckpt_dir, "config.json"))
        self.st = SafeTensors(ckpt_dir)
        if self.st.has("model.language_model.embed_tokens.weight"):
            prefix = "model.language_model."
        elif self.st.has("model.embed_tokens.weight"):
            prefix = "model."
        else:
            raise ValueError(f"unrecognised checkpoint layout in {ckpt_dir}")
        c = self.cfg
        cc = _Cfg(c.hidden, c.intermediate, c.n_layers, c.vocab, c.eps, c.n_heads, c.n_kv_heads, c.head_dim,
                  c.rotary_dim, c.rope_theta, c.conv_kernel, c.lin_k_heads, c.lin_v_heads, c.lin_k_dim, c.lin_v_dim)
        kinds = (C.c_int * c.n_layers)(*[0 if k == "linear" else 1 for k in c.layer_kinds])
        self._h = lib().oracle_model_new(C.byref(cc), kinds)
        lib().oracle_model_kv_bf16(self._h, 1 if kv_bf16 else 0, float(kv_perturb))
        self._keep = []
        embed = self.st.mat16(prefix + "embed_tokens.weight")
        if embed.shape[0] < c.vocab or embed.shape[1] != c.hidden:
            raise ValueError("embedding shape does not match config")
        self._set(-1, 1, embed)
        if self.st.has("lm_head.weight") and not c.tie_embeddings:
            self.lm_head = self.st.mat16("lm_head.weight")
        else:
            self.lm_head = embed
        self._set(-1, 2, self.lm_head)
        self.embed = embed
        for i, kind in enumerate(c.layer_kinds):
            pre = f"{prefix}layers.{i}."
            for name, slot in _MATS.items():
                if (kind == "linear") == name.startswith("linear_attn") or name.startswith("mlp"):
                    self._set(i, slot, self.st.mat16(pre + name))
            for name, slot in _VECS.items():
                want = name.startswith("linear_attn") if kind == "linear" else name.startswith("self_attn")
                if want or name.endswith("layernorm.weight"):
                    self._set(i, slot, self.st.f32s(pre + name))
        self._set(-1, 42, self.st.f32s(prefix + "norm.weight"))

    def _set(self, layer: int, slot: int, arr: np.ndarray):
        arr = np.ascontiguousarray(arr)
        self._keep.append(arr)
        is_bf16 = 1 if arr.dtype == np.uint16 else 0
        if not is_bf16:
            arr = np.ascontiguousarray(arr, dtype=np.float32)
            self._keep.append(arr)
        rows, cols = (arr.shape[0], arr.shape[1]) if arr.ndim == 2 else (1, arr.size)
        rc = lib().oracle_model_set(self._h, layer, slot, _p(arr), is_bf16, rows, cols)
        if rc != 0:
            raise RuntimeError(f"oracle_model_set({layer}, {slot}) -> {rc}")

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.oracle_model_free(self._h)
            self._h = None

    def neuron_sigma(self):
        """analysis.rs:129-201 (through the lens when one is set): (sigma [layers * intermediate], unembedding mean
        [hidden], m_scale)."""
        sig = np.zeros(self.cfg.n_layers * self.cfg.intermediate, np.float32)
        mean = np.zeros(self.cfg.hidden, np.float32)
        ms = lib().oracle_neuron_sigma(self._h, _p(sig), _p(mean))
        return sig, mean, float(ms)

    def set_lens(self, maps: dict, kind: str, target_layer: int):
        """A loaded lens (lens.rs:10-54): maps {layer: [hidden][hidden] uint16 bits}, kind "f16" or "bf16"."""
        d, L = self.cfg.hidden, self.cfg.n_layers
        self._lens = {l: np.ascontiguousarray(m, dtype=np.uint16).reshape(d, d) for l, m in maps.items()}
        ptrs = (C.c_void_p * L)(*[self._lens[l].ctypes.data if l in self._lens else None for l in range(L)])
        lib().oracle_lens_set(self._h, ptrs, L, 0 if kind == "f16" else 1, int(target_layer))

    def clear_lens(self):
        lib().oracle_lens_clear(self._h)
        self._lens = {}

    def lens_logits(self, layer: int, vecs: np.ndarray) -> np.ndarray:
        """analysis.rs:28-34: [n][vocab] logits of residual-basis vectors [n][hidden] at `layer`."""
        x = np.ascontiguousarray(vecs, dtype=np.float32).reshape(-1, self.cfg.hidden)
        out = np.zeros((x.shape[0], self.cfg.vocab), np.float32)
        lib().oracle_lens_logits(self._h, int(layer), _p(x), x.shape[0], _p(out))
        return out

    def neuron_logits(self, neurons) -> np.ndarray:
        """analysis.rs:37-67: [n][vocab] logits of the write directions of (layer, neuron) pairs."""
        ls = np.ascontiguousarray([l for l, _ in neurons], np.int32)
        ns = np.ascontiguousarray([n for _, n in neurons], np.int32)
        out = np.zeros((len(neurons), self.cfg.vocab), np.float32)
        lib().oracle_neuron_logits(self._h, _p(ls), _p(ns), len(neurons), _p(out))
        return out

    def search(self, tokens, mean: np.ndarray, sigma: np.ndarray, limit: int):
        """analysis.rs:213-251: the top `limit` hits (layer, neuron, sign, z) for the token ids."""
        t = np.ascontiguousarray(tokens, np.uint32)
        mean = np.ascontiguousarray(mean, np.float32)
        sigma = np.ascontiguousarray(sigma, np.float32)
        hl, hn, hs = (np.zeros(limit, np.int32) for _ in range(3))
        hz = np.zeros(limit, np.float32)
        k = lib().oracle_search(self._h, _p(t), len(t), _p(mean), _p(sigma), int(limit), _p(hl), _p(hn), _p(hs),
                                _p(hz))
        return [(int(hl[i]), int(hn[i]), int(hs[i]), float(hz[i])) for i in range(k)]

    def new_cache(self) -> "Cache":
        return Cache(lib().oracle_cache_new(self._h))

    def seeded_cache(self, pos: int, seed: int = 0) -> "Cache":
        """A cache standing at position `pos` with generator-filled states, conv windows and `pos` key/value rows
        (oracle_cache_seed): a timing aid for decode at long contexts without a prefill."""
        c = self.new_cache()
        lib().oracle_cache_seed(self._h, c._h, pos, seed)
        return c

    def col_norms_down(self, layer: int) -> np.ndarray:
        """||W_down[:, n]|| per neuron, in f64 like kernels.rs:79-103, returned as f32."""
        prefix = "model.language_model." if self.st.has("model.language_model.embed_tokens.weight") else "model."
        w = self.st.f32s(f"{prefix}layers.{layer}.mlp.down_proj.weight").reshape(self.cfg.hidden, -1)
        return np.sqrt((w.astype(np.float64) ** 2).sum(0)).astype(np.float32)

    def forward(self, seqs, want_logits=True, act_scale=None, track_max=None):
        """seqs: list of dicts {cache, tokens, plan?, gate?, frames?(bool), resid?(bool)}.

        Returns (logits [nseq, vocab] or None, frames list, resid list)."""
        n = len(seqs)
        arr = (_Seq * max(n, 1))()
        keep = []
        frames, resid = [], []
        for i, s in enumerate(seqs):
            toks = np.ascontiguousarray(s["tokens"], dtype=np.uint32)
            keep.append(toks)
            fr = np.zeros((len(toks), self.cfg.n_layers * self.cfg.intermediate), np.int8) if s.get("frames") else None
            rs = np.zeros((len(toks), self.cfg.n_layers * self.cfg.hidden), np.uint16) if s.get("resid") else None
            frames.append(fr)
            resid.append(rs)
            plan = s.get("plan")
            arr[i] = _Seq(s["cache"]._h, _p(toks) if len(toks) else None, len(toks),
                          plan._h if plan is not None else None,
                          s["gate"]._h if plan is not None else None,
                          _p(fr) if fr is not None else None, _p(rs) if rs is not None else None)
        logits = np.zeros((n, self.lm_head.shape[0]), np.float32) if want_logits else None
        sc = np.ascontiguousarray(act_scale, dtype=np.float32) if act_scale is not None else None
        lib().oracle_forward(self._h, arr, n, _p(sc) if sc is not None else None,
                             _p(track_max) if track_max is not None else None, 1 if want_logits else 0,
                             _p(logits) if logits is not None else None)
        return logits, frames, resid


class Cache:
    def __init__(self, h):
        self._h = h

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.oracle_cache_free(self._h)
            self._h = None

    def clone(self) -> "Cache":
        return Cache(lib().oracle_cache_clone(self._h))

    @property
    def pos(self) -> int:
        return lib().oracle_cache_pos(self._h)

    def read(self, layer: int, which: str) -> np.ndarray:
        code = {"state": 0, "conv": 1, "k": 2, "v": 3}[which]
        n = lib().oracle_cache_read(self._h, layer, code, None, 0)
        out = np.zeros(n, np.float32)
        lib().oracle_cache_read(self._h, layer, code, _p(out), n)
        return out


class Plan:
    def __init__(self, n_layers: int):
        self._h = lib().oracle_plan_new(n_layers)
        self.n_gates = 0

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.oracle_plan_free(self._h)
            self._h = None

    def begin(self, st: "GateState", rows: int):
        lib().oracle_plan_begin(self._h, st._h, rows)

    def apply(self, layer: int, acts: np.ndarray, n: int, st: "GateState"):
        assert acts.dtype == np.float32 and acts.flags["C_CONTIGUOUS"]
        lib().oracle_plan_apply(self._h, layer, _p(acts), n, acts.size // n, st._h)


class GateState:
    def __init__(self):
        self._h = lib().oracle_gate_state_new()

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.oracle_gate_state_free(self._h)
            self._h = None

    def open(self, g: int) -> bool:
        return bool(lib().oracle_gate_state_open(self._h, g))

    def score(self, g: int) -> float:
        return float(lib().oracle_gate_state_score(self._h, g))

    def partial(self, g: int) -> np.ndarray:
        """Detector sums of gate g per row of the latest pass."""
        n = lib().oracle_gate_state_partial(self._h, g, None, 0)
        out = np.zeros(n, np.float32)
        if n:
            lib().oracle_gate_state_partial(self._h, g, _p(out), n)
        return out


MODE = {"add": 1, "mul": 2, "set": 3}


def compile_plan(ivs, n_layers: int, n_neurons: int, unit) -> Plan:
    """steering.rs:118-139. ivs: dicts {layer, neuron, mode, value, enabled?, gate?: {detectors, threshold}}."""
    plan = Plan(n_layers)
    for iv in ivs:
        if not iv.get("enabled", True) or not (iv["layer"] < n_layers and iv["neuron"] < n_neurons):
            continue
        mode = iv.get("mode", "add")
        if mode == "add":  # f32 value x f32 unit, as steering.rs:123 multiplies them
            value = np.float32(iv["value"]) * np.float32(unit(iv["layer"], iv["neuron"]))
        else:
            value = iv["value"]
        value = float(np.float32(value))
        gi = -1
        g = iv.get("gate")
        if g and g.get("detectors"):
            dets = [d for d in g["detectors"] if d["layer"] < n_layers and d["neuron"] < n_neurons]
            last = max([0] + [d["layer"] for d in dets])
            gi = lib().oracle_plan_add_gate(plan._h, float(np.float32(g["threshold"])), last)
            for d in dets:
                lib().oracle_plan_add_detector(plan._h, gi, d["layer"], d["neuron"], float(d.get("weight", 1.0)))
            plan.n_gates += 1
        lib().oracle_plan_add_op(plan._h, iv["layer"], iv["neuron"], MODE[mode], value, gi)
    return plan

