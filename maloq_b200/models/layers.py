"""Equivariant building blocks of the eSEN/HELM backbone.

Module and parameter names follow the reference so that ``state_dict`` keys match
(``helm/nn/*.py``); the arithmetic is routed through :mod:`maloq_b200.ops`, which runs
the sm_100a kernels on CUDA tensors and the PyTorch definitions on CPU tensors.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from .. import ops
from .so3 import CoefficientMapping, l_expand_index


class GaussianSmearing(nn.Module):
    """exp(coeff (d - mu_k)^2) on ``num_gaussians`` centres in [start, stop].

    Reference ``helm/nn/radial.py:44-60``; ``offset`` is a persistent buffer.
    """

    def __init__(self, start=0.0, stop=5.0, num_gaussians=50, basis_width_scalar=1.0):
        super().__init__()
        self.num_output = num_gaussians
        offset = torch.linspace(start, stop, num_gaussians)
        self.coeff = -0.5 / (basis_width_scalar * (offset[1] - offset[0])).item() ** 2
        self.register_buffer("offset", offset)

    def forward(self, dist):
        return torch.exp(self.coeff * (dist.view(-1, 1) - self.offset.view(1, -1)) ** 2)


class PolynomialEnvelope(nn.Module):
    """1 + a d^p + b d^(p+1) + c d^(p+2) for d < 1, else 0 (reference ``radial.py:21-41``)."""

    def __init__(self, exponent: int = 5):
        super().__init__()
        p = float(exponent)
        self.p, self.a, self.b, self.c = p, -(p + 1) * (p + 2) / 2, p * (p + 2), -p * (p + 1) / 2

    def forward(self, d):
        env = 1 + self.a * d ** self.p + self.b * d ** (self.p + 1) + self.c * d ** (self.p + 2)
        return torch.where(d < 1, env, torch.zeros_like(d))


class SphericalBesselBasis(nn.Module):
    def __init__(self, num_radial: int, cutoff: float):
        super().__init__()
        self.norm_const = math.sqrt(2 / cutoff**3)
        self.frequencies = nn.Parameter(torch.pi * torch.arange(1, num_radial + 1, dtype=torch.float32))

    def forward(self, d_scaled):
        return self.norm_const / d_scaled[:, None] * torch.sin(self.frequencies * d_scaled[:, None])


class EnvelopedBesselBasis(nn.Module):
    """Envelope x spherical Bessel basis (reference ``radial.py:87-112``)."""

    def __init__(self, num_radial: int, cutoff: float):
        super().__init__()
        self.inv_cutoff = 1 / cutoff
        self.envelope = PolynomialEnvelope()
        self.rbf = SphericalBesselBasis(num_radial, cutoff)
        self.num_output = num_radial

    def forward(self, d):
        ds = d * self.inv_cutoff
        return self.envelope(ds)[:, None] * self.rbf(ds)


class RadialMLP(nn.Module):
    """Linear -> LayerNorm -> SiLU stack, last layer linear (reference ``radial.py:115-142``).

    ``net`` indices 0,1,3,4,6 hold the parameters for a 3-entry channel list, matching the
    reference's checkpoint keys.  The LayerNorm+SiLU pairs run as one fused kernel.
    """

    def __init__(self, channels_list):
        super().__init__()
        mods = []
        cin = channels_list[0]
        for i in range(1, len(channels_list)):
            mods.append(nn.Linear(cin, channels_list[i], bias=True))
            cin = channels_list[i]
            if i == len(channels_list) - 1:
                break
            mods.append(nn.LayerNorm(channels_list[i]))
            mods.append(nn.SiLU())
        self.net = nn.Sequential(*mods)

    def forward(self, x):
        mods = list(self.net)
        i = 0
        while i < len(mods):
            lin = mods[i]
            x = ops.linear(x, lin.weight, lin.bias)
            if i + 1 < len(mods) and isinstance(mods[i + 1], nn.LayerNorm):
                ln = mods[i + 1]
                x = ops.layernorm_silu(x, ln.weight, ln.bias, ln.eps)
                i += 3
            else:
                i += 1
        return x


class SO3_Linear(nn.Module):
    """Per-degree channel mixing, weight [(L+1), Cout, Cin], bias on l = 0 (``so3_layers.py:14-48``)."""

    def __init__(self, in_features: int, out_features: int, lmax: int):
        super().__init__()
        self.in_features, self.out_features, self.lmax = in_features, out_features, lmax
        self.weight = nn.Parameter(torch.empty(lmax + 1, out_features, in_features))
        bound = 1 / math.sqrt(in_features)
        nn.init.uniform_(self.weight, -bound, bound)
        self.bias = nn.Parameter(torch.zeros(out_features))
        self.register_buffer("expand_index", l_expand_index(lmax))

    def forward(self, x):
        return ops.so3_linear(x, self.weight, self.bias, self.lmax)


class GateActivation(nn.Module):
    """SiLU on the scalar entry, tanh(gate) times every other entry of the same degree.

    ``outer_dim='l'`` gates an l-major [(L+1)^2] layout; ``'m'`` the m-major edge-frame
    layout (reference ``helm/nn/activation.py:12-77``).
    """

    def __init__(self, lmax: int, mmax: int, num_channels: int, outer_dim="l", mapping: CoefficientMapping | None = None):
        super().__init__()
        self.lmax, self.mmax, self.num_channels, self.outer_dim = lmax, mmax, num_channels, outer_dim
        if outer_dim == "l":
            idx = []
            for l in range(1, lmax + 1):
                idx += [l - 1] * min(2 * l + 1, 2 * mmax + 1)
            expand_index = torch.tensor(idx, dtype=torch.long)
        else:
            assert mapping is not None
            expand_index = mapping.gate_expand_index()
        self.register_buffer("expand_index", expand_index)

    def forward(self, gating_scalars, x):
        return ops.gate(gating_scalars, x, self.expand_index, self.lmax)


class EquivariantRMSNorm(nn.Module):
    """Degree-balanced equivariant RMS norm with l=0 centring (``rms_norm_sh``).

    out = (x - [mean_c x_00 on l=0]) * rsqrt(mean_c sum_i w_i x_i^2 + eps) * affine_weight[l]
    (+ affine_bias on l=0), with w_i = 1 / ((2l+1)(L+1)).  Reference
    ``helm/nn/layer_norm.py:230-338``.
    """

    def __init__(self, lmax: int, num_channels: int, eps: float = 1e-5):
        super().__init__()
        self.lmax, self.num_channels, self.eps = lmax, num_channels, eps
        self.affine_weight = nn.Parameter(torch.ones(lmax + 1, num_channels))
        self.affine_bias = nn.Parameter(torch.zeros(num_channels))
        self.register_buffer("expand_index", l_expand_index(lmax))
        bw = torch.zeros((lmax + 1) ** 2, 1)
        for l in range(lmax + 1):
            bw[l * l : l * l + 2 * l + 1] = 1.0 / (2 * l + 1)
        self.register_buffer("balance_degree_weight", bw / (lmax + 1))

    def forward(self, x, residual=None):
        """norm(x), or (norm(x + residual), x + residual) when ``residual`` is given."""
        return ops.rms_norm_sh(x, self.affine_weight, self.affine_bias, self.balance_degree_weight, self.eps, residual)


def get_normalization_layer(norm_type: str, lmax: int, num_channels: int):
    if norm_type != "rms_norm_sh":
        raise ValueError(f"unsupported norm_type {norm_type!r} (this framework implements 'rms_norm_sh')")
    return EquivariantRMSNorm(lmax, num_channels)


class SO2_m_Conv(nn.Module):
    """Linear over the (l, channel) entries of one |m| > 0 pair (reference ``so2_layers.py:19-67``).

    ``fc.weight`` is [2 Nh, K] = [W_r; W_i].  Applied to the (+m, -m) rows (x0, x1) it
    gives out_+ = W_r x0 - W_i x1 and out_- = W_r x1 + W_i x0; :meth:`pair_weight`
    writes that as one [2Nh, 2K] real matrix [[W_r, -W_i], [W_i, W_r]] so the pair is one
    GEMM over the concatenated rows.
    """

    def __init__(self, m: int, sphere_channels: int, m_output_channels: int, lmax: int, mmax: int):
        super().__init__()
        self.m = m
        n_coef = lmax - m + 1
        self.out_channels_half = m_output_channels * n_coef
        self.fc = nn.Linear(n_coef * sphere_channels, 2 * self.out_channels_half, bias=False)
        self.fc.weight.data.mul_(1 / math.sqrt(2))

    def pair_weight(self):
        w = self.fc.weight
        h = self.out_channels_half
        wr, wi = w[:h], w[h:]
        return torch.cat([torch.cat([wr, -wi], dim=1), torch.cat([wi, wr], dim=1)], dim=0)


class SO2_Convolution(nn.Module):
    """Per-|m| linear maps in the edge frame, optionally modulated by a radial MLP.

    Input/output are m-major [E, R, C].  With ``extra_m0_output_channels`` the m = 0 map
    also emits gating scalars, returned separately.  Reference ``so2_layers.py:70-214``.
    """

    def __init__(self, sphere_channels, m_output_channels, lmax, mmax, mapping: CoefficientMapping,
                 internal_weights=True, edge_channels_list=None, extra_m0_output_channels=None):
        super().__init__()
        self.sphere_channels, self.m_output_channels = sphere_channels, m_output_channels
        self.lmax, self.mmax = lmax, mmax
        self.m_size = list(mapping.m_size)
        self.extra_m0_output_channels = extra_m0_output_channels
        n_m0 = (lmax + 1) * sphere_channels
        out_m0 = m_output_channels * (lmax + 1) + (extra_m0_output_channels or 0)
        self.fc_m0 = nn.Linear(n_m0, out_m0, bias=True)
        n_rad = n_m0
        self.so2_m_conv = nn.ModuleList()
        for m in range(1, mmax + 1):
            self.so2_m_conv.append(SO2_m_Conv(m, sphere_channels, m_output_channels, lmax, mmax))
            n_rad += self.so2_m_conv[-1].fc.in_features
        self.rad_func = None
        if not internal_weights:
            chans = list(edge_channels_list) + [int(n_rad)]
            self.rad_func = RadialMLP(chans)

    def gemm_weights(self):
        """[fc_m0.weight, pair weight m=1, ...] - one GEMM per |m| block."""
        return [self.fc_m0.weight] + [c.pair_weight() for c in self.so2_m_conv]

    def forward(self, x, x_edge, rad=None):
        if self.rad_func is not None and rad is None:
            rad = self.rad_func(x_edge)
        out, extra = ops.so2_conv(x, rad, self.gemm_weights(), self.fc_m0.bias, self.m_size,
                                  self.extra_m0_output_channels or 0, self.m_output_channels)
        if self.extra_m0_output_channels:
            return out, extra
        return out
