"""Import-compatible module of the reference package (maloq.helm.esen_block); the implementation lives in
:mod:`maloq_b200.models.backbone`."""

from maloq_b200.models.backbone import Edgewise, SpectralAtomwise, eSEN_Block  # noqa: F401
