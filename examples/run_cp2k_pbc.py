"""Graph-partitioned training on a periodic CP2K structure (one structure split over GPUs).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/run_cp2k_pbc.py

``dbpath`` holds structure directories with ``structure.xyz`` (``Cell:`` or ``Lattice=``
header) and ``hamiltonian.csr`` (CP2K sparse dump), optionally ``overlap.csr`` + ``cp2k.out``
for the Fermi-level shift.  ``structure_index`` picks the directory.
"""
import torch

from maloq.train_utils import loss, training_workflow

config = {
    "dataset_name": "cp2k", "dbpath": "cp2k_data", "structure_index": 0, "basis_name": "dzvp_like",
    "distribute_graphs": True, "partition_type": "linear-edgewise", "message_type": "source-target-message",
    "output_folder": "outputs_cp2k", "run_name": "cp2k", "train_or_eval": "train", "num_epochs": 10,
    "dtype": torch.float32, "lr_init": 1e-4, "optimizer_type": "adamw", "loss_target": "fock_matrix",
    "train_loss_fxn": loss.rmse_mse_padded_loss, "test_loss_fxn": loss.l1_unpadded_loss,
    "reduce_node": True, "reduce_node_intra": True, "l_embedding_dim": 128, "num_distance_basis": 128,
    "num_mp_layers": 6, "mmax": 2, "rcut_orbitals": 4.0, "rcut_gaussian": 8.0,
    "edge_chunk": None,  # set (e.g. 131072) for structures whose edges exceed device memory
}

if __name__ == "__main__":
    training_workflow.TrainingWorkflow(config).run()
