"""Import-compatible module of the reference package (maloq.fock_utils.domain_decomp); the implementation lives in
:mod:`maloq_b200.parallel.partition`."""

from maloq_b200.parallel.partition import Domain, decompose, halo_volume, local_domain, partition  # noqa: F401
