"""The reference package's import paths resolve to this framework's implementations."""


def test_reference_import_paths():
    from maloq.dataset_utils.get_loader import read_cp2k_matrix
    from maloq.dataset_utils.nablaDFT_dataset_utils import HamiltonianDatabase
    from maloq.fock_utils.domain_decomp import decompose
    from maloq.fock_utils.matrix2labels_kernels import SparseBlockMatrix
    from maloq.fock_utils.utils_tensor_decomp import e3TensorDecomp
    from maloq.helm.common.so3 import CoefficientMapping
    from maloq.helm.esen_block import eSEN_Block
    from maloq.helm.esen_osh import Fock_Irreps_Head, eSEN_Backbone
    from maloq.helm.nn.layer_norm import EquivariantRMSNormArraySphericalHarmonicsV2
    from maloq.helm.nn.so2_layers import SO2_Convolution
    from maloq.train_utils.splittrainer import SplitTrainer
    from maloq.train_utils.utils_compute import split_indices
    from maloq_b200.core.wigner3j import BasisTransform
    from maloq_b200.data.labels import BlockSparseMatrix
    from maloq_b200.data.readers import NablaDFTDatabase, read_cp2k_csr
    from maloq_b200.models import backbone, heads, layers
    from maloq_b200.train.trainer import SplitTrainer as ST

    assert e3TensorDecomp is BasisTransform and SparseBlockMatrix is BlockSparseMatrix
    assert HamiltonianDatabase is NablaDFTDatabase and read_cp2k_matrix is read_cp2k_csr
    assert eSEN_Backbone is backbone.eSEN_Backbone and eSEN_Block is backbone.eSEN_Block
    assert Fock_Irreps_Head is heads.Fock_Irreps_Head and SO2_Convolution is layers.SO2_Convolution
    assert EquivariantRMSNormArraySphericalHarmonicsV2 is layers.EquivariantRMSNorm
    assert SplitTrainer is ST and callable(decompose) and callable(split_indices) and CoefficientMapping


def test_reference_data_tool_import_paths():
    from maloq.dataset_utils.ASEDataset import ASEDataset, distribute_data
    from maloq.dataset_utils.compute_lin_ref_nabla import linear_energy_references
    from maloq.dataset_utils.get_scale_shift import scale_shift_table
    from maloq.dataset_utils.omol_csh_58k_dataset_utils import OMolCSH58kDatabase
    from maloq.fock_utils.get_energy_from_fock import hf_energy, write_density_cube
    from maloq.fock_utils.utils_orca_out import get_fock_size, sort_by_l

    assert all(callable(f) for f in (ASEDataset, distribute_data, linear_energy_references, scale_shift_table,
                                     OMolCSH58kDatabase, hf_energy, write_density_cube, get_fock_size, sort_by_l))
