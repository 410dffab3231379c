"""Zonotope symbolic expressions (reference: constraintflow/lib/symexp.py:14-273).

Kept importable for generated programs (`from constraintflow.lib.symexp import *`).  The
zonotope state of zono.cf is held by the network driver on the device (cf_deeppoly_run with
CF_RELAX_ZONO: symbol coefficients one row per noise symbol); Flow.flow runs the whole
program there, so these objects are never computed with on the host."""


def get_new_eps(*args, **kwargs):
    raise NotImplementedError("zonotope programs run as a whole in the network driver (Flow.flow); the "
                              "op-by-op symbol algebra is not provided")


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
