"""Import-compatible module of the reference package (maloq.fock_utils.reorder); the implementation lives in
:mod:`maloq_b200.parallel.partition`."""

from maloq_b200.parallel.partition import (  # noqa: F401
    PARTITIONERS, partition_approx_neighbors, partition_bruteforce, partition_greedy, partition_local_optimal,
    partition_rcb, partition_slab, partition_surface_volume, partition_worst_case,
)
