"""Import-compatible module of the reference package (maloq.helm.nn.so3_layers); the implementation lives in
:mod:`maloq_b200.models.layers`."""

from maloq_b200.models.layers import SO3_Linear  # noqa: F401
