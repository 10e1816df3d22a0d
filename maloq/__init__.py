"""Import-compatible entry points of the reference package (``maloq.train_utils``,
``maloq.core.config``, ``maloq.cli``), implemented by :mod:`maloq_b200`."""
