"""Import-compatible module of the reference package (maloq.helm.nn.radial); the implementation lives in
:mod:`maloq_b200.models.layers`."""

from maloq_b200.models.layers import (  # noqa: F401
    EnvelopedBesselBasis, GaussianSmearing, PolynomialEnvelope, RadialMLP, SphericalBesselBasis,
)
