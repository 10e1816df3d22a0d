"""Graph-partitioned training on an amorphous Si/O supercell (one structure split over GPUs).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/run_sio2_partitioned.py
Set ``train_or_eval`` to ``"infer"`` to write each rank's block-sparse Hamiltonian shard.
"""
import torch

from maloq.train_utils import loss, training_workflow

config = {
    "dataset_name": "synthetic_sio2", "num_atoms": 20000, "distribute_graphs": True, "partition_type": "slab",
    "halo_transport": None,  # NVLink peer halo on GPUs, collective otherwise
    "output_folder": "outputs_sio2", "run_name": "sio2", "train_or_eval": "train", "num_epochs": 10,
    "dtype": torch.float32, "lr_init": 1e-4, "optimizer_type": "adamw", "loss_target": "fock_matrix",
    "train_loss_fxn": loss.rmse_mse_padded_loss, "test_loss_fxn": loss.l1_unpadded_loss,
    "reduce_node": True, "reduce_node_intra": True, "l_embedding_dim": 128, "num_distance_basis": 128,
    "num_mp_layers": 6, "mmax": 4, "rcut_orbitals": 4.0, "rcut_gaussian": 8.0, "message_type": "source-target",
}

if __name__ == "__main__":
    training_workflow.TrainingWorkflow(config).run()
