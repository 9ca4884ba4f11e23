"""frontend: PyTorch -> anvil.graph (capture + quantize) and the host numerics behind it.

    q = from_torch(module, (x_example,), calib, headroom=1.5)   # capture + quantize (anvil/frontend/__init__.py:17-19)

torch is imported lazily, so this package imports without it.
"""
import importlib

from .numerics import fixed_point, prove_no_overflow

_LAZY = {"capture": "capture", "FGraph": "capture", "FNode": "capture", "UnsupportedOpError": "capture",
         "quantize": "quantize", "Quantized": "quantize"}


def __getattr__(name):
    if name in _LAZY:
        mod = importlib.import_module(f"{__name__}.{_LAZY[name]}")
        return getattr(mod, name)
    raise AttributeError(name)


def from_torch(module, example_inputs, calib_inputs, headroom=1.5, **kw):
    """capture(module, example_inputs) then quantize(..., calib_inputs, headroom, **kw)."""
    from .capture import capture
    from .quantize import quantize
    return quantize(capture(module, example_inputs), calib_inputs, headroom, **kw)


__all__ = ["FGraph", "FNode", "Quantized", "UnsupportedOpError", "capture", "fixed_point", "from_torch",
           "prove_no_overflow", "quantize"]
