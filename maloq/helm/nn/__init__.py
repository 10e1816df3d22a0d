"""Import-compatible module of the reference package (maloq.helm.nn); the implementation lives in
:mod:`maloq_b200.models.layers`."""
