"""Import-compatible module of the reference package (maloq.helm.esen_osh); the implementation lives in
:mod:`maloq_b200.models`."""

from maloq_b200.models.backbone import eSEN_Backbone  # noqa: F401
from maloq_b200.models.heads import (  # noqa: F401
    Fock_Irreps_Head, HELM_Energy_Head, HELM_Force_Head, HELM_Simple_Force_Head,
)
