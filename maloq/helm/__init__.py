"""Import-compatible module of the reference package (maloq.helm); the implementation lives in
:mod:`maloq_b200.models`."""
