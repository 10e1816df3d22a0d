"""Import-compatible module of the reference package (maloq.helm.common.rotation); the implementation lives in
:mod:`maloq_b200.core.sph`."""

from maloq_b200.core.sph import (  # noqa: F401
    J_matrices, edge_euler_angles, euler_matrix, wigner_D, wigner_D_from_matrix,
)
