from maloq_b200.train.workflow import TrainingWorkflow  # noqa: F401
