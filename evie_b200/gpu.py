"""GpuModel: Python view of the full-model C ABI, with the method set of evie-core's GPU backend
(crates/evie-core/src/gpu/mod.rs: new, forward, set_ops, reset_slot, set_scale, track_max, read_max), plus the
gated steering plans (set_plan, gate_state, reset_gates) and per-slot samplers (set_sampler) of the CPU engine."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import EvieError, capi, lib

MODES = {"add": 1, "mul": 2, "set": 3}
# evie_seq as a numpy record (the layout of capi.Seq), for sequence tables built by array operations
_SEQ_DTYPE = np.dtype({"names": ["slot", "pos0", "tokens", "n_tokens"], "formats": ["<i4", "<i4", "<u8", "<i4"],
                       "offsets": [capi.Seq.slot.offset, capi.Seq.pos0.offset, capi.Seq.tokens.offset,
                                   capi.Seq.n_tokens.offset], "itemsize": C.sizeof(capi.Seq)})


@dataclass
class GpuSeq:
    """One sequence in a forward call (gpu/mod.rs:147-154)."""
    slot: int
    pos0: int
    tokens: np.ndarray


@dataclass
class GpuOut:
    """gpu/mod.rs:156-163, plus the greedy token of each sequence."""
    logits: np.ndarray | None = None                  # [n_seqs, vocab] f32
    frames: np.ndarray | None = None                  # [rows, layers*neurons] i8
    resid: np.ndarray | None = None                   # [rows, layers*hidden] f16
    next_tokens: np.ndarray = field(default_factory=lambda: np.zeros(0, np.uint32))


class GpuModel:
    def __init__(self, ckpt_dir: str, max_ctx: int, slots: int = 2, max_rows: int = 128, device: int = 0):
        L = lib()
        h = C.c_void_p()
        rc = L.evie_create(ckpt_dir.encode(), device, slots, max_ctx, max_rows, C.byref(h))
        if rc != 0:
            raise EvieError(rc, (L.evie_last_global_error() or b"").decode())
        self._h = h
        info = capi.ModelInfo()
        self._check(L.evie_info(self._h, C.byref(info)))
        self.info = info
        self.layers, self.neurons, self.hidden, self.vocab = info.n_layers, info.intermediate, info.hidden, info.vocab
        self.slots, self.max_ctx, self.max_rows = info.slots, info.max_ctx, info.max_rows
        self._n_gates: dict[int, int] = {}

    def _check(self, rc: int):
        if rc != 0:
            raise EvieError(rc, (lib().evie_last_error(self._h) or b"").decode())

    def close(self):
        if getattr(self, "_h", None):
            lib().evie_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, seqs, want_logits: bool = True, capture: bool = False, out: GpuOut | None = None) -> GpuOut:
        n = len(seqs)
        arr = (capi.Seq * max(n, 1))()
        keep = []
        rows = 0
        for i, s in enumerate(seqs):
            t = np.ascontiguousarray(s.tokens, dtype=np.uint32)
            keep.append(t)
            arr[i] = capi.Seq(s.slot, s.pos0, t.ctypes.data if t.size else None, t.size)
            rows += t.size
        return self._forward_table(C.addressof(arr), n, rows, want_logits, capture, out)

    def forward_batch(self, slots, pos0, tokens, counts=None, want_logits: bool = True, capture: bool = False,
                      out: GpuOut | None = None) -> GpuOut:
        """forward() for a batch given as arrays: sequence i runs in slot slots[i] from position pos0[i] on
        counts[i] tokens (1 each when counts is None), all tokens concatenated in sequence order in `tokens`. The
        same evie_forward call; the sequence table is built by array operations, not by a loop over GpuSeq
        objects, which keeps the host's share of a decode step small (one token per sequence, tens of sequences)."""
        slots = np.asarray(slots, np.int32).ravel()
        n = slots.size
        pos0 = np.broadcast_to(np.asarray(pos0, np.int32), (n,))
        counts = np.ones(n, np.int32) if counts is None else np.asarray(counts, np.int32).ravel()
        tokens = np.ascontiguousarray(tokens, np.uint32).ravel()
        if counts.size != n or (counts < 0).any() or int(counts.sum()) != tokens.size:
            raise ValueError("forward_batch: counts must give one non-negative count per slot, summing to len(tokens)")
        tab = np.zeros(max(n, 1), _SEQ_DTYPE)
        first = np.zeros(n, np.uint64)
        np.cumsum(counts[:-1], out=first[1:])
        tab["slot"][:n] = slots
        tab["pos0"][:n] = pos0
        tab["n_tokens"][:n] = counts
        tab["tokens"][:n] = np.where(counts > 0, np.uint64(tokens.ctypes.data) + 4 * first, 0)
        return self._forward_table(tab.ctypes.data, n, tokens.size, want_logits, capture, out)

    def _forward_table(self, table: int, n: int, rows: int, want_logits: bool, capture: bool,
                       out: GpuOut | None) -> GpuOut:
        """evie_forward on a table of n evie_seq records at address `table` holding `rows` tokens in all (the
        caller keeps the table and the token arrays alive across the call)."""
        o = out or GpuOut()
        if want_logits and (o.logits is None or o.logits.shape != (n, self.vocab)):
            o.logits = np.empty((n, self.vocab), np.float32)
        if capture:
            if o.frames is None or o.frames.shape != (rows, self.layers * self.neurons):
                o.frames = np.empty((rows, self.layers * self.neurons), np.int8)
            if o.resid is None or o.resid.shape != (rows, self.layers * self.hidden):
                o.resid = np.empty((rows, self.layers * self.hidden), np.float16)
        if o.next_tokens.shape != (n,):
            o.next_tokens = np.empty(n, np.uint32)
        p = lambda a: a.ctypes.data if a is not None else None  # noqa: E731
        self._check(lib().evie_forward(self._h, table, n, int(want_logits), int(capture),
                                       p(o.logits) if want_logits else None, p(o.frames) if capture else None,
                                       p(o.resid) if capture else None, p(o.next_tokens)))
        return o

    def decode_greedy(self, seqs, steps: int, capture: bool = False, frames=None, resid=None) -> np.ndarray:
        """evie_decode_greedy: `steps` greedy steps on the device. Returns the tokens [steps, n_seqs]."""
        n = len(seqs)
        arr = (capi.Seq * n)()
        keep = []
        for i, s in enumerate(seqs):
            t = np.ascontiguousarray(s.tokens, dtype=np.uint32)
            keep.append(t)
            arr[i] = capi.Seq(s.slot, s.pos0, t.ctypes.data, t.size)
        out = np.empty((steps, n), np.uint32)
        p = lambda a: a.ctypes.data if a is not None else None  # noqa: E731
        self._check(lib().evie_decode_greedy(self._h, arr, n, steps, out.ctypes.data, int(capture), p(frames),
                                             p(resid)))
        return out

    def profile(self, on: bool):
        self._check(lib().evie_profile(self._h, int(on)))

    def profile_read(self) -> dict:
        """{group: (ms, launches)} accumulated since profiling was switched on."""
        out = {}
        i = 0
        while True:
            name, ms, n = C.c_char_p(), C.c_double(), C.c_int64()
            cnt = lib().evie_profile_read(self._h, i, C.byref(name), C.byref(ms), C.byref(n))
            if i >= cnt:
                break
            out[name.value.decode()] = (ms.value, n.value)
            i += 1
        return out

    def stream_ptr(self) -> int:
        """The cudaStream_t the context enqueues its work on (for CUDA-event timing)."""
        return lib().evie_stream(self._h) or 0

    def set_ops(self, slot: int, ops):
        """ops: iterable of (layer, neuron, mode 1/2/3 or 'add'/'mul'/'set', value)."""
        ops = list(ops)
        arr = (capi.Op * max(len(ops), 1))()
        for i, (l, nn, m, v) in enumerate(ops):
            arr[i] = capi.Op(l, nn, MODES.get(m, m) if isinstance(m, str) else m, v)
        self._check(lib().evie_set_ops(self._h, slot, arr, len(ops)))
        self._n_gates[slot] = 0

    def set_plan(self, slot: int, plan):
        """A compiled steering.Plan with its detector gates; closes the slot's gates (Plan::new_state)."""
        ops = (capi.PlanOp * max(len(plan.ops), 1))(*[capi.PlanOp(*o) for o in plan.ops])
        th = np.ascontiguousarray(plan.thresholds, dtype=np.float32)
        dets = (capi.Detector * max(len(plan.detectors), 1))(*[capi.Detector(*d) for d in plan.detectors])
        self._check(lib().evie_set_plan(self._h, slot, ops, len(plan.ops), th.ctypes.data if th.size else None,
                                        th.size, dets, len(plan.detectors)))
        self._n_gates[slot] = th.size

    def gate_state(self, slot: int) -> tuple[np.ndarray, np.ndarray]:
        """(open [n_gates] bool, score [n_gates] f32) of the slot's gates (GateState::open / ::score)."""
        n = self._n_gates.get(slot, 0)
        op = np.zeros(max(n, 1), np.int32)
        sc = np.zeros(max(n, 1), np.float32)
        self._check(lib().evie_gate_state(self._h, slot, op.ctypes.data, sc.ctypes.data, max(n, 1)))
        return op[:n].astype(bool), sc[:n]

    def set_sampler(self, slot: int, temperature: float = 0.0, top_p: float = 1.0, min_p: float = 0.0,
                    repetition_penalty: float = 1.0, seed: int = 0):
        """Sampler::new(SampleParams) for the slot (sampling.rs:27-29); the defaults are greedy."""
        sp = capi.SampleParams(temperature, top_p, min_p, repetition_penalty, seed)
        self._check(lib().evie_set_sampler(self._h, slot, C.byref(sp)))

    def top_active(self, k: int = 20) -> np.ndarray:
        """[rows, k] flat neuron indices (layer * neurons + neuron) of the k largest |frame| entries of every row the
        last capturing call left on the device, as evie's top_active tool ranks them (equal |q|: lower index)."""
        out = np.empty((max(self.max_rows, 1), k), np.int32)
        rows = C.c_int()
        self._check(lib().evie_read_top_active(self._h, k, out.ctypes.data, C.byref(rows)))
        return out[:rows.value].copy()

    def neuron_sigma(self):
        """analysis.rs:129-201 through the current lens: (sigma [layers * neurons], unembedding mean [hidden],
        m_scale)."""
        sig = np.empty(self.layers * self.neurons, np.float32)
        mean = np.empty(self.hidden, np.float32)
        ms = C.c_float()
        self._check(lib().evie_neuron_sigma(self._h, sig.ctypes.data, sig.size, mean.ctypes.data, C.byref(ms)))
        return sig, mean, ms.value

    def set_lens(self, lens):
        """Copies a lens (evie_b200.lens.Lens) to the device for the analysis calls; None drops it (logit lens)."""
        if lens is None:
            self._check(lib().evie_clear_lens(self._h))
            return
        d = self.hidden
        keep = {l: np.ascontiguousarray(m, np.uint16).reshape(d, d) for l, m in lens.maps.items()}
        ptrs = (C.c_void_p * self.layers)(*[keep[l].ctypes.data if l in keep else None for l in range(self.layers)])
        self._check(lib().evie_set_lens(self._h, ptrs, self.layers, 0 if lens.kind == "f16" else 1,
                                        int(lens.target_layer)))

    def lens_logits(self, layer: int, vecs: np.ndarray) -> np.ndarray:
        """analysis.rs:28-34: [n][vocab] logits of residual-basis vectors [n][hidden] living at `layer`."""
        x = np.ascontiguousarray(vecs, np.float32).reshape(-1, self.hidden)
        out = np.empty((x.shape[0], self.vocab), np.float32)
        self._check(lib().evie_lens_logits(self._h, int(layer), x.ctypes.data, x.shape[0], out.ctypes.data))
        return out

    def neuron_logits(self, neurons) -> np.ndarray:
        """analysis.rs:37-67: [n][vocab] logits of the write directions of (layer, neuron) pairs."""
        ls = np.ascontiguousarray([l for l, _ in neurons], np.int32)
        ns = np.ascontiguousarray([n for _, n in neurons], np.int32)
        out = np.empty((len(neurons), self.vocab), np.float32)
        self._check(lib().evie_neuron_logits(self._h, ls.ctypes.data, ns.ctypes.data, len(neurons), out.ctypes.data))
        return out

    def search_scores(self, tokens, mean: np.ndarray, sigma: np.ndarray):
        """analysis.rs:213-240: per-neuron best z of each pole, ([layers][neurons], [layers][neurons])."""
        t = np.ascontiguousarray(tokens, np.uint32)
        mean = np.ascontiguousarray(mean, np.float32)
        sigma = np.ascontiguousarray(sigma, np.float32)
        up = np.empty((self.layers, self.neurons), np.float32)
        dn = np.empty((self.layers, self.neurons), np.float32)
        self._check(lib().evie_search_scores(self._h, t.ctypes.data, t.size, mean.ctypes.data, sigma.ctypes.data,
                                             up.ctypes.data, dn.ctypes.data))
        return up, dn

    def reset_gates(self, slot: int):
        self._check(lib().evie_reset_gates(self._h, slot))

    def reset_slot(self, slot: int):
        self._check(lib().evie_reset_slot(self._h, slot))

    def set_scale(self, scale: np.ndarray):
        s = np.ascontiguousarray(scale, dtype=np.float32)
        self._check(lib().evie_set_scale(self._h, s.ctypes.data, s.size))

    def track_max(self, on: bool):
        self._check(lib().evie_track_max(self._h, int(on)))

    def read_max(self) -> np.ndarray:
        out = np.empty(self.layers * self.neurons, np.float32)
        self._check(lib().evie_read_max(self._h, out.ctypes.data, out.size))
        return out
