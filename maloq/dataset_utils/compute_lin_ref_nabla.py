"""Import-compatible module of the reference package (maloq.dataset_utils.compute_lin_ref_nabla); the
implementation lives in :mod:`maloq_b200.data.tools`."""

from maloq_b200.data.tools import dataset_statistics, linear_energy_references, pooled_molecules  # noqa: F401
