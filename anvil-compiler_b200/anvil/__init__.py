"""anvil (B200 build): the `cuda` execution target for Anvil's int8-quantized transformer graphs.

    import anvil
    cm = anvil.compile(module, (x_example,), calib)       # anvil.driver.compile -> CompiledModel
    cm.run(x, "cuda").output                              # hand-written sm_100a kernels via libanvil_cuda.so

Mirrors the reference entry point (anvil/__init__.py:9-12): `compile` is imported lazily so `import anvil` stays
light.
"""


def compile(*args, **kw):  # noqa: A001  (the public entry point shadows the builtin inside this package only)
    """anvil.driver.compile."""
    from .driver import compile as _compile
    return _compile(*args, **kw)


def __getattr__(name):
    if name in ("CudaParams", "CompiledModel", "RunOutput"):
        from . import driver
        return getattr(driver, name)
    raise AttributeError(name)


__all__ = ["compile", "CudaParams", "CompiledModel", "RunOutput"]
