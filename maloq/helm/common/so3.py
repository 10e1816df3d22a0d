"""Import-compatible module of the reference package (maloq.helm.common.so3); the implementation lives in
:mod:`maloq_b200.models.so3`."""

from maloq_b200.models.so3 import CoefficientMapping  # noqa: F401
