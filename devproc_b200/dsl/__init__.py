"""``@kernel`` DSL: decorator, symbolic tensors, op functions and type markers."""

from .kernel import KernelContext, KernelTensor, kernel, parse_ir

__all__ = ["KernelContext", "KernelTensor", "kernel", "parse_ir"]
