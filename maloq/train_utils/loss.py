from maloq_b200.train.loss import *  # noqa: F401,F403
