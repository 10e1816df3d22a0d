"""Import-compatible module of the reference package (maloq.dataset_utils); the implementation lives in
:mod:`maloq_b200.data`."""
