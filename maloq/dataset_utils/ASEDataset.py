"""Import-compatible module of the reference package (maloq.dataset_utils.ASEDataset); the implementation lives in
:mod:`maloq_b200.data.asedb`."""

from maloq_b200.data.asedb import ASEAtomsData, ASEDataset, distribute_data, get_rank_range  # noqa: F401
