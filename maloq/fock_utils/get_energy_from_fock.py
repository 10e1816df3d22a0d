"""Import-compatible module of the reference package (maloq.fock_utils.get_energy_from_fock); the implementation lives in
:mod:`maloq_b200.eval.electronic`."""

from maloq_b200.eval.electronic import (  # noqa: F401
    closed_shell_density, orbitals, orthogonalizer, summary, total_energy,
)
