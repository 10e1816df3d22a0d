"""Import-compatible module of the reference package (maloq.fock_utils.basis_sets); the implementation lives in
:mod:`maloq_b200.data.basis_sets`."""

from maloq_b200.data.basis_sets import *  # noqa: F401,F403
