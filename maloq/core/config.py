from maloq_b200.core.config import *  # noqa: F401,F403
