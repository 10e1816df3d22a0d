"""Training on a nablaDFT Hamiltonian database (SQLite file given by ``dbpath``)."""
import sys

import torch

from maloq.train_utils import loss, training_workflow

config = {
    "dataset_name": "nablaDFT", "dbpath": sys.argv[1] if len(sys.argv) > 1 else "train_2k.db",
    "num_structures": 2000, "output_folder": "outputs_nabla", "run_name": "nabla", "batch_size": 8,
    "num_epochs": 100, "dtype": torch.float32, "lr_init": 1e-4, "optimizer_type": "adamw",
    "scheduler_type": "plateau", "patience": 10, "threshold": 1e-8, "loss_target": "fock_matrix",
    "train_loss_fxn": loss.rmse_mse_padded_loss, "test_loss_fxn": loss.l1_unpadded_loss,
    "reduce_node": True, "reduce_node_intra": True, "l_embedding_dim": 128, "num_distance_basis": 128,
    "num_mp_layers": 3, "rcut_orbitals": 8.0, "rcut_gaussian": 16.0,
}

if __name__ == "__main__":
    training_workflow.TrainingWorkflow(config).run()
