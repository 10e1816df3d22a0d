"""``maloq --config run.yaml [--print-effective-config]`` (reference ``cli/main.py:13-37``)."""

from __future__ import annotations

import argparse
import json


def main(argv=None):
    ap = argparse.ArgumentParser(prog="maloq", description="Train/evaluate/infer Hamiltonian models")
    ap.add_argument("--config", required=True, help="YAML/TOML/JSON config (nested or flat)")
    ap.add_argument("--print-effective-config", action="store_true", help="print the resolved config and exit")
    args = ap.parse_args(argv)
    from ..core.config import MaloqConfig

    cfg = MaloqConfig.from_file(args.config)
    if args.print_effective_config:
        print(json.dumps(cfg.model_dump(), indent=2, default=str))
        return 0
    from ..train.workflow import TrainingWorkflow

    TrainingWorkflow(cfg.to_workflow_config()).run()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
