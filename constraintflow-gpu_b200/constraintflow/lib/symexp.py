"""Zonotope symbolic expressions (reference: constraintflow/lib/symexp.py:14-273).

Kept importable for generated programs (`from constraintflow.lib.symexp import *`); the
DeepZ family of certifiers that computes with them is not run by this runtime."""


def get_new_eps(*args, **kwargs):
    raise NotImplementedError("zonotope (DeepZ) certifiers are not run by this runtime")


class SymExpSparse:
    count = 0

    def __init__(self, network, mat, const):
        self.network = network
        self.mat = mat
        self.const = const

    def get_mat(self, *args, **kwargs):
        return self.mat

    def get_const(self, *args, **kwargs):
        return self.const
