"""Neuron interventions and their compiled plans: the host half of evie-core's steering module
(crates/evie-core/src/steering.rs), feeding evie_set_plan.

An intervention edits one MLP neuron's activation at the input of down_proj (steering.rs:1-5): Add adds
`value` doses (one dose = the layer's dose unit, supplied by the caller as steering.rs:117 takes it), Mul
multiplies, Set clamps. An optional Gate makes it conditional: the gate opens, and stays open for the rest of the
conversation, once the weighted sum of its detector neurons' activations exceeds its threshold on some token
(steering.rs:29-34). The device applies the compiled plan inside the SwiGLU epilogue (evie_set_plan)."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable

import numpy as np

MODE_CODE = {"add": 1, "mul": 2, "set": 3}


def _f32(x) -> float:
    return float(np.float32(x))


@dataclass
class Detector:
    """steering.rs:21-27 (weight defaults to 1.0)."""
    layer: int
    neuron: int
    weight: float = 1.0


@dataclass
class Gate:
    """steering.rs:29-34."""
    detectors: list[Detector]
    threshold: float


@dataclass
class Intervention:
    """steering.rs:36-50 (mode defaults to add, enabled to true)."""
    layer: int
    neuron: int
    value: float
    mode: str = "add"
    enabled: bool = True
    label: str = ""
    gate: Gate | None = None

    @staticmethod
    def add(layer: int, neuron: int, dose: float) -> "Intervention":
        """steering.rs:59-61."""
        return Intervention(layer, neuron, dose)


@dataclass
class Plan:
    """The compiled plan (steering.rs:97-104) in the flat form evie_set_plan takes:
    ops      (layer, neuron, mode code, value, gate index or -1), in intervention order;
    thresholds one per gate;
    detectors (gate, layer, neuron, weight), in compile order (per gate, in the gate's detector order)."""
    ops: list[tuple[int, int, int, float, int]] = field(default_factory=list)
    thresholds: list[float] = field(default_factory=list)
    detectors: list[tuple[int, int, int, float]] = field(default_factory=list)
    last_layer: list[int] = field(default_factory=list)

    @property
    def n_gates(self) -> int:
        return len(self.thresholds)

    def is_empty(self) -> bool:
        """steering.rs:141-143."""
        return not self.ops

    @staticmethod
    def compile(ivs: list[Intervention], n_layers: int, n_neurons: int,
                unit: Callable[[int, int], float]) -> "Plan":
        """steering.rs:118-139: enabled, in-range interventions; Add values become value x unit(layer, neuron)
        in f32; a gate with at least one detector gets the next gate index, keeps its in-range detectors and
        decides at the deepest of their layers (0 when none is in range)."""
        plan = Plan()
        for iv in ivs:
            if not (iv.enabled and 0 <= iv.layer < n_layers and 0 <= iv.neuron < n_neurons):
                continue
            if iv.mode not in MODE_CODE:
                raise ValueError(f"unknown mode {iv.mode!r}")
            if iv.mode == "add":
                value = _f32(np.float32(iv.value) * np.float32(unit(iv.layer, iv.neuron)))
            else:
                value = _f32(iv.value)
            gi = -1
            if iv.gate is not None and iv.gate.detectors:
                gi = plan.n_gates
                last = 0
                for d in iv.gate.detectors:
                    if 0 <= d.layer < n_layers and 0 <= d.neuron < n_neurons:
                        plan.detectors.append((gi, d.layer, d.neuron, _f32(d.weight)))
                        last = max(last, d.layer)
                plan.thresholds.append(_f32(iv.gate.threshold))
                plan.last_layer.append(last)
            plan.ops.append((iv.layer, iv.neuron, MODE_CODE[iv.mode], value, gi))
        return plan
