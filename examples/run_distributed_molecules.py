"""Graph-parallel training on molecules: every batch of molecules is one graph (their disjoint
union) split over all ranks, with halo exchange between the ranks' domains.

    torchrun --nproc-per-node 4 --master-addr 127.0.0.1 examples/run_distributed_molecules.py [nabla.db]

Without a database argument it trains on synthetic drug-like molecules with teacher targets.
"""
import sys

from maloq.train_utils import loss, training_workflow

config = {
    "dataset_name": "nablaDFT" if len(sys.argv) > 1 else "synthetic_druglike",
    "dbpath": sys.argv[1] if len(sys.argv) > 1 else None, "num_structures": 64,
    "distribute_graphs": True, "partition_type": "rcb", "batch_size": 4,
    "output_folder": "outputs_distributed_molecules", "run_name": "dist_mol", "num_epochs": 10,
    "lr_init": 1e-4, "loss_target": "fock_matrix", "train_loss_fxn": loss.rmse_mse_padded_loss,
    "test_loss_fxn": loss.l1_unpadded_loss, "l_embedding_dim": 128, "num_distance_basis": 128,
    "num_mp_layers": 4, "rcut_orbitals": 3.0, "rcut_gaussian": 6.0, "mmax": 2,
}

if __name__ == "__main__":
    training_workflow.TrainingWorkflow(config).run()
