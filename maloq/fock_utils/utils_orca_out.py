"""Import-compatible module of the reference package (maloq.fock_utils.utils_orca_out); the implementation lives in
:mod:`maloq_b200.data.readers`."""

from maloq_b200.data.readers import CONVENTIONS, read_orca_output, reorder_orbitals  # noqa: F401
