"""maloq_b200: equivariant Hamiltonian learning (eSEN/HELM backbone + Fock heads) for NVIDIA
B200 (sm_100a).  PyTorch is the framework layer; hot ops are sm_100a CUDA kernels
(``maloq_b200/ops/csrc``); multi-GPU paths use NCCL plus in-kernel NVLink peer access."""

__version__ = "0.1.0"
