"""Quantization of a captured float graph (placeholder: filled in with the nanoGPT frontend)."""
from dataclasses import dataclass, field


@dataclass
class Quantized:
    module: object
    consts: dict
    scales: dict
    bounds: dict
    graph: object = None
    syms: dict = field(default_factory=dict)
