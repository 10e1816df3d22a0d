"""Import-compatible module of the reference package (maloq.dataset_utils.get_scale_shift); the implementation lives
in :mod:`maloq_b200.data.tools` (``scale_shift_table``) and :mod:`maloq_b200.data.targets` (``ScaleShift``)."""

from maloq_b200.data.readers import fermi_energy as get_fermi_energy  # noqa: F401
from maloq_b200.data.targets import ScaleShift  # noqa: F401
from maloq_b200.data.tools import scale_shift_table  # noqa: F401
