"""anvil.ir: the anvil.graph dialect (xDSL-free) and its generic MLIR text form.

    text = print_ir(module); module2 = parse_ir(text)       # textual round trip (anvil/ir/__init__.py:22-32)
"""
from . import graph
from .graph import GraphBuilder, Module, QTensorType, VerifyException
from .text import ParseError, parse_ir, print_ir


def module(*funcs):
    return Module(list(funcs)).verify()


__all__ = ["graph", "GraphBuilder", "Module", "QTensorType", "VerifyException", "ParseError", "parse_ir", "print_ir",
           "module"]
