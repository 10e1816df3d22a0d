"""Import-compatible module of the reference package (maloq.helm.nn.layer_norm); the implementation lives in
:mod:`maloq_b200.models.layers`. The default
``rms_norm_sh`` normalisation is ``EquivariantRMSNorm``."""

from maloq_b200.models.layers import EquivariantRMSNorm, get_normalization_layer  # noqa: F401

EquivariantRMSNormArraySphericalHarmonicsV2 = EquivariantRMSNorm
