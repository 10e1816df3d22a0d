"""Import-compatible module of the reference package (maloq.dataset_utils.get_loader); the implementation lives in
:mod:`maloq_b200.data`."""

from maloq_b200.data.batch import batches_by_atoms, batches_by_count, collate  # noqa: F401
from maloq_b200.data.readers import fermi_energy, read_cp2k_csr, read_periodic_xyz  # noqa: F401

read_cp2k_matrix = read_cp2k_csr
get_fermi_energy = fermi_energy
