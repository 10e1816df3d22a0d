"""Import-compatible module of the reference package (maloq.dataset_utils.omol_csh_58k_dataset_utils); the
implementation lives in :mod:`maloq_b200.data.omol`."""

from maloq_b200.data.omol import OMolCSH58kDatabase, restore_orca_diffuse_order, save_keys_manifest  # noqa: F401
