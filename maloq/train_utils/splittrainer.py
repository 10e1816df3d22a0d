"""Import-compatible module of the reference package (maloq.train_utils.splittrainer); the implementation lives in
:mod:`maloq_b200.train.trainer`."""

from maloq_b200.train.trainer import SplitTrainer  # noqa: F401
