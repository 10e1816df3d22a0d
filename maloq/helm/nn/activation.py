"""Import-compatible module of the reference package (maloq.helm.nn.activation); the implementation lives in
:mod:`maloq_b200.models.layers`."""

from maloq_b200.models.layers import GateActivation  # noqa: F401
