"""The torch side of the cuda target: a PyTorch module becomes a quantized anvil.graph module in two stages.

`capture` exports the module with torch.export and matches its ATen graph into a small float op graph (FGraph);
`quantize` calibrates that graph on sample inputs and lowers it to the integer IR with its constants. `from_torch`
chains the two, which is what `anvil.compile` calls for a torch module. The host-side constant builders and the
int32 overflow proof live in `numerics`. torch is imported only inside the functions that need it.
"""
from .capture import FGraph, FNode, UnsupportedOpError, capture
from .numerics import fixed_point, prove_no_overflow
from .quantize import Quantized, quantize

__all__ = ["FGraph", "FNode", "Quantized", "UnsupportedOpError", "capture", "fixed_point", "from_torch",
           "prove_no_overflow", "quantize"]


def from_torch(module, example_inputs, calib_inputs, headroom=1.5, **kw) -> Quantized:
    """Capture `module` on `example_inputs`, then quantize the captured graph on `calib_inputs` (the reference's
    from_torch, anvil/frontend/__init__.py:17-19); extra keywords go to quantize."""
    return quantize(capture(module, example_inputs), calib_inputs, headroom, **kw)
