"""Data-parallel training on synthetic drug-like molecules (def2-SVP-like basis).

    python examples/run_synthetic_druglike.py                      # one GPU
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/run_synthetic_druglike.py
"""
import torch

from maloq.train_utils import loss, training_workflow

config = {
    "dataset_name": "synthetic_druglike", "num_structures": 256, "output_folder": "outputs_druglike",
    "run_name": "druglike", "train_or_eval": "train", "batch_size": 32, "num_epochs": 10,
    "dtype": torch.float32, "lr_init": 1e-4, "optimizer_type": "adam", "scheduler_type": "cosine", "eta_min": 1e-8,
    "loss_target": "fock_matrix", "train_loss_fxn": loss.rmse_mse_padded_loss, "test_loss_fxn": loss.l1_unpadded_loss,
    "reduce_node": True, "reduce_node_intra": True, "reduce_edge": False,
    "l_embedding_dim": 128, "num_distance_basis": 128, "num_mp_layers": 6, "mmax": 2,
    "rcut_orbitals": 3.0, "rcut_gaussian": 6.0, "gaussian_width": 1.0, "save_frequency": 5,
}

if __name__ == "__main__":
    training_workflow.TrainingWorkflow(config).run()
