"""Import-compatible module of the reference package (maloq.helm.nn.so2_layers); the implementation lives in
:mod:`maloq_b200.models.layers`."""

from maloq_b200.models.layers import SO2_Convolution, SO2_m_Conv  # noqa: F401
