"""Import-compatible module of the reference package (maloq.dataset_utils.nablaDFT_dataset_utils); the implementation lives in
:mod:`maloq_b200.data.readers`."""

from maloq_b200.data.readers import NablaDFTDatabase, load_nabladft  # noqa: F401

HamiltonianDatabase = NablaDFTDatabase
