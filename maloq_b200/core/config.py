"""Typed run configuration (reference ``core/config.py``) - YAML/TOML/JSON, nested or flat.

Sections: dataset, execution, split, model, optimization, loss, checkpoint, runtime.
Unknown keys are kept (``extra="allow"``).  A flat legacy file (all keys at top level, as
``examples/nabla_minimal.yaml``) is sorted into sections by key name.
:meth:`MaloqConfig.to_workflow_config` returns the flat dict ``TrainingWorkflow`` takes,
with loss names mapped to functions and dtype strings to torch dtypes.

The accepted values are the superset of the reference's two entry paths:
``optimizer_type`` in {adam, adamw, muon}; ``train_or_eval`` in {train, eval, infer}.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Literal

from pydantic import BaseModel, ConfigDict

LossName = Literal["mse_padded_loss", "l1_padded_loss", "rmse_padded_loss", "rmse_mse_padded_loss",
                   "combined_padded_loss", "mse_unpadded_loss", "weighted_irrep_mse_loss", "l1_unpadded_loss",
                   "geometric_mean_loss", "combined_unpadded_loss"]


class _Section(BaseModel):
    model_config = ConfigDict(extra="allow")


class DatasetConfig(_Section):
    dataset_name: str = "synthetic_druglike"
    dbpath: Any = ""
    output_folder: str = "outputs"
    run_name: str = "run"
    open_shell: bool = False
    num_structures: int = 64


class ExecutionConfig(_Section):
    train_or_eval: Literal["train", "eval", "infer"] = "train"
    train_backbone: bool = True
    train_head: bool = True
    compute_total_energy: bool = False


class SplitConfig(_Section):
    num_train: int = 0
    num_val: int = 0
    num_test: int = 0
    batch_size: int = 1
    shuffle: bool = False
    distribute_graphs: bool = False
    partition_type: str | None = None
    dist_backend: str = "nccl"


class ModelConfig(_Section):
    wigner_backend: str = "cuda"
    activation_checkpointing: bool = False
    l_embedding_dim: int = 128
    num_distance_basis: int = 128
    num_mp_layers: int = 3
    rcut_orbitals: float = 8.0
    rcut_gaussian: float = 16.0
    gaussian_width: float = 1.0
    reduce_edge: bool = False
    reduce_node: bool = True
    reduce_node_intra: bool = True
    mmax: int | None = None


class OptimizationConfig(_Section):
    num_epochs: int = 1
    lr_init: float = 1e-4
    optimizer_type: Literal["adam", "adamw", "muon"] = "adam"
    weight_decay: float = 0.0
    scheduler_type: Literal["cosine", "plateau"] = "cosine"
    eta_min: float = 1e-8
    patience: int = 100
    threshold: float = 1e-8
    step_every_epoch: bool = False


class LossConfig(_Section):
    loss_target: Literal["fock_matrix", "density_matrix", "energies", "forces"] = "fock_matrix"
    train_loss: LossName = "rmse_mse_padded_loss"
    test_loss: LossName = "l1_unpadded_loss"
    scale_and_shift: bool = False


class CheckpointConfig(_Section):
    save_frequency: int = 10
    restart_backbone: bool = False
    restart_head: bool = False
    restart_optimizer: bool = False
    backbone_checkpoint: str = "backbone.pt"
    head_checkpoint: str = "head.pt"


class RuntimeConfig(_Section):
    dtype: Literal["float32", "float64", "bfloat16"] = "float32"


SECTIONS = {"dataset": DatasetConfig, "execution": ExecutionConfig, "split": SplitConfig, "model": ModelConfig,
            "optimization": OptimizationConfig, "loss": LossConfig, "checkpoint": CheckpointConfig,
            "runtime": RuntimeConfig}


class MaloqConfig(BaseModel):
    model_config = ConfigDict(extra="allow")
    dataset: DatasetConfig = DatasetConfig()
    execution: ExecutionConfig = ExecutionConfig()
    split: SplitConfig = SplitConfig()
    model: ModelConfig = ModelConfig()
    optimization: OptimizationConfig = OptimizationConfig()
    loss: LossConfig = LossConfig()
    checkpoint: CheckpointConfig = CheckpointConfig()
    runtime: RuntimeConfig = RuntimeConfig()

    @classmethod
    def from_mapping(cls, raw: dict) -> "MaloqConfig":
        raw = dict(raw)
        if not any(k in SECTIONS for k in raw):
            raw = coerce_flat(raw)
        return cls(**raw)

    @classmethod
    def from_file(cls, path) -> "MaloqConfig":
        p = Path(path)
        text = p.read_text()
        if p.suffix in (".yaml", ".yml"):
            import yaml

            raw = yaml.safe_load(text) or {}
        elif p.suffix == ".toml":
            import tomllib

            raw = tomllib.loads(text)
        elif p.suffix == ".json":
            raw = json.loads(text)
        else:
            raise ValueError(f"unsupported config format {p.suffix!r}")
        return cls.from_mapping(raw)

    def to_workflow_config(self) -> dict:
        import torch

        from ..train import loss as L

        flat = {}
        for name in SECTIONS:
            flat.update(getattr(self, name).model_dump())
        flat.update({k: v for k, v in (self.model_extra or {}).items()})
        flat["train_loss_fxn"] = L.get_loss(flat.pop("train_loss"))
        flat["test_loss_fxn"] = L.get_loss(flat.pop("test_loss"))
        flat["dtype"] = {"float32": torch.float32, "float64": torch.float64, "bfloat16": torch.bfloat16}[flat["dtype"]]
        return flat


def coerce_flat(raw: dict) -> dict:
    """Sort flat (legacy) keys into sections; keys no section declares stay top-level extras."""
    out: dict = {k: {} for k in SECTIONS}
    for k, v in raw.items():
        for name, model in SECTIONS.items():
            if k in model.model_fields:
                out[name][k] = v
                break
        else:
            if k in ("train_loss_fxn", "test_loss_fxn"):
                out["loss"][k.replace("_fxn", "")] = getattr(v, "__name__", v)
            else:
                out[k] = v
    return out
