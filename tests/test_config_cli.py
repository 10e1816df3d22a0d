"""Config loading (flat and nested YAML), CLI --print-effective-config, CPU training run."""
import json
import os

from maloq_b200.cli import main as cli
from maloq_b200.core.config import MaloqConfig

EX = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "examples")


def test_flat_and_nested_yaml():
    flat = MaloqConfig.from_file(os.path.join(EX, "nabla_minimal.yaml"))
    assert flat.model.num_mp_layers == 4 and flat.split.batch_size == 8 and flat.model.mmax == 2
    nested = MaloqConfig.from_file(os.path.join(EX, "druglike_nested.yaml"))
    wf = nested.to_workflow_config()
    assert wf["num_mp_layers"] == 6 and wf["train_loss_fxn"].__name__ == "rmse_mse_padded_loss"


def test_cli_print_effective_config(capsys):
    cli.main(["--config", os.path.join(EX, "nabla_minimal.yaml"), "--print-effective-config"])
    out = json.loads(capsys.readouterr().out)
    assert out["dataset"]["dataset_name"] == "synthetic_small"


def test_cli_trains_on_cpu(tmp_path):
    import yaml

    cfg = yaml.safe_load(open(os.path.join(EX, "nabla_minimal.yaml")))
    cfg.update(output_folder=str(tmp_path), num_structures=10, num_epochs=1, l_embedding_dim=8, num_mp_layers=1,
               device="cpu")
    p = tmp_path / "c.yaml"
    p.write_text(yaml.safe_dump(cfg))
    cli.main(["--config", str(p)])
    assert (tmp_path / "backbone.pt").exists() and (tmp_path / "head.pt").exists()
