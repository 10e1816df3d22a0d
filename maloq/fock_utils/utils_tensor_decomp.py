"""Import-compatible module of the reference package (maloq.fock_utils.utils_tensor_decomp); the implementation lives in
:mod:`maloq_b200.core`. ``e3TensorDecomp``
is :class:`BasisTransform` (``get_H`` / ``get_net_out``); ``make_output_irreps`` is
:func:`make_label_layout`."""

from maloq_b200.core.irreps import make_label_layout  # noqa: F401
from maloq_b200.core.wigner3j import BasisTransform, l1l2_to_l3s, wigner_3j  # noqa: F401

e3TensorDecomp = BasisTransform
make_output_irreps = make_label_layout
