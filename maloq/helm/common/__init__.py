"""Import-compatible module of the reference package (maloq.helm.common); the implementation lives in
:mod:`maloq_b200.core`."""
