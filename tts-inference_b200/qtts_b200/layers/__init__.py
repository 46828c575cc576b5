from .linear import LinearBase, MergedLinear, QuantMethod, iter_linears

__all__ = ["LinearBase", "MergedLinear", "QuantMethod", "iter_linears"]
