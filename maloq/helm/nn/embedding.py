"""Import-compatible module of the reference package (maloq.helm.nn.embedding); the implementation lives in
:mod:`maloq_b200.models.backbone`."""

from maloq_b200.models.backbone import EdgeDegreeEmbedding  # noqa: F401
