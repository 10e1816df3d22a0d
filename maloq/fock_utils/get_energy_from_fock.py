"""Import-compatible module of the reference package (maloq.fock_utils.get_energy_from_fock); the implementation
lives in :mod:`maloq_b200.eval.electronic` and :mod:`maloq_b200.eval.integrals` (own one-electron integrals, the
Hartree-Fock energy functional, density cube and xyz files)."""

from maloq_b200.eval.electronic import (  # noqa: F401
    closed_shell_density, orbitals, orthogonalizer, summary, total_energy,
)
from maloq_b200.eval.integrals import (  # noqa: F401
    hf_energy, one_electron_integrals, write_density_cube, write_xyz,
)
