from maloq_b200.train import loss, workflow as training_workflow  # noqa: F401
from maloq_b200.train import trainer as splittrainer  # noqa: F401
