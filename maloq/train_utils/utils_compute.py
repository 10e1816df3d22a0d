"""Import-compatible module of the reference package (maloq.train_utils.utils_compute); the implementation lives in
:mod:`maloq_b200.parallel.dist`."""

from maloq_b200.parallel.dist import cleanup_process_group, setup_env, split_indices  # noqa: F401
