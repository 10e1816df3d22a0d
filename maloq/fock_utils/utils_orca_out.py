"""Import-compatible module of the reference package (maloq.fock_utils.utils_orca_out); the implementation lives in
:mod:`maloq_b200.data.readers`.  Functions the reference names differently are bound to its names."""

from maloq_b200.data.readers import (  # noqa: F401
    CONVENTIONS, charge_and_multiplicity_from_path, homo_lumo_energies, orbital_count, read_finalms, read_orca_output,
    reorder_orbitals, sort_by_l,
)

extract_charge_and_spin_from_path = charge_and_multiplicity_from_path
get_finalms = read_finalms
get_fock_size = orbital_count
