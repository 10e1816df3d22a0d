"""OMol-CSH-58k Hamiltonians (HDF5 file + ``<file>.keys.json`` manifest, def2-TZVPD; the ORCA
diffuse-shell order is corrected on load).  Reading HDF5 needs h5py.  A folder of ASE ``.db``
files (``dbpath`` a directory) is read the same way with each rank loading only its rows.

    python examples/run_omol_csh.py       # edit dbpath below first
"""
import torch

from maloq.train_utils import loss, training_workflow

config = {
    "dataset_name": "omol_csh_58k",
    "dbpath": "omol_csh_58k.h5",
    "output_folder": "outputs_omol_csh",
    "run_name": "omol_csh",
    "open_shell": False,
    "train_or_eval": "train",
    "num_train": 50000,
    "num_val": 1000,
    "batch_size": 8,
    "reduce_edge": False,
    "reduce_node": True,
    "reduce_node_intra": True,
    "num_epochs": 100,
    "dtype": torch.float32,
    "lr_init": 5e-4,
    "optimizer_type": "adamw",
    "weight_decay": 1e-4,
    "scheduler_type": "cosine",
    "loss_target": "fock_matrix",
    "train_loss_fxn": loss.rmse_mse_padded_loss,
    "test_loss_fxn": loss.l1_unpadded_loss,
    "scale_and_shift": True,
    "l_embedding_dim": 128,
    "num_distance_basis": 128,
    "num_mp_layers": 4,
    "mmax": 2,
    # radius per atom: the graph joins atoms closer than 2 * rcut_orbitals
    "rcut_orbitals": 3.0,
    "rcut_gaussian": 6.0,
    "gaussian_width": 1.0,
}


def main():
    training_workflow.TrainingWorkflow(config).run()


if __name__ == "__main__":
    main()
