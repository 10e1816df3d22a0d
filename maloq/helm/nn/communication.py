"""Import-compatible module of the reference package (maloq.helm.nn.communication); the implementation lives in
:mod:`maloq_b200.parallel`. The halo
exchange is a :class:`HaloPlan` (collective) or a :class:`PeerHalo` (NVLink peer memory)."""

from maloq_b200.parallel.halo import HaloPlan, partition_batch  # noqa: F401
from maloq_b200.parallel.peer_halo import PeerHalo  # noqa: F401
