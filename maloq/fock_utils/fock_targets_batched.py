"""Import-compatible module of the reference package (maloq.fock_utils.fock_targets_batched); the implementation lives in
:mod:`maloq_b200.data.targets`. The
target pipeline is :class:`FockLabeler` (+ :class:`Teacher` for synthetic data)."""

from maloq_b200.data.targets import FockLabeler, ScaleShift, Teacher, attach_targets  # noqa: F401
