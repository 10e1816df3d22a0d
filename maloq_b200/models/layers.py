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

    def forward(self, x, out_dtype=None):
        """``out_dtype``: dtype of the last layer's output on the kernel path (the edge kernels
        read the radial modulation as bf16)."""
        mods = list(self.net)
        i = 0
        while i < len(mods):
            lin = mods[i]
            last = i == len(mods) - 1
            x = ops.linear(x, lin.weight, lin.bias, out_dtype=out_dtype if last else None)
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

    def forward(self, x, out_dtype=None, residual=None):
        """``residual`` is added to the output (fused on the kernel path); ``out_dtype``: bf16
        output on the kernel path when the consumer is another GEMM."""
        return ops.so3_linear(x, self.weight, self.bias, self.lmax, out_dtype, residual)


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

    def forward(self, x, residual=None, out_dtype=None):
        """norm(x), or (norm(x + residual), x + residual) when ``residual`` is given.  On the
        kernel path ``out_dtype`` = bf16 stores norm(.) as bf16 (the sum stays fp32)."""
        return ops.rms_norm_sh(x, self.affine_weight, self.affine_bias, self.balance_degree_weight, self.eps, residual,
                               out_dtype)


class _ResidualNorm(nn.Module):
    """``forward(x, residual=None)`` convention of the norms: with a residual, returns
    (norm(x + residual), x + residual)."""

    def forward(self, x, residual=None, out_dtype=None):
        if residual is None:
            return self.normalize(x)
        s = x + residual
        return self.normalize(s), s


class EquivariantLayerNormArray(_ResidualNorm):
    """Per-degree equivariant layer norm (``layer_norm``): each l block is divided by the RMS
    over its (2l+1) components ("component") or their sum ("norm") and the channels; l = 0 is
    centred over the channels first; per-l affine weight, l = 0 bias.  Reference
    ``helm/nn/layer_norm.py:47-119``."""

    def __init__(self, lmax: int, num_channels: int, eps: float = 1e-5, affine: bool = True,
                 normalization: str = "component"):
        super().__init__()
        if normalization not in ("norm", "component"):
            raise ValueError(normalization)
        self.lmax, self.num_channels, self.eps, self.affine = lmax, num_channels, eps, affine
        self.normalization = normalization
        if affine:
            self.affine_weight = nn.Parameter(torch.ones(lmax + 1, num_channels))
            self.affine_bias = nn.Parameter(torch.zeros(num_channels))
        else:
            self.register_parameter("affine_weight", None)
            self.register_parameter("affine_bias", None)
        self.register_buffer("_deg", l_expand_index(lmax), persistent=False)

    def normalize(self, x):
        L = self.lmax
        x0 = x[:, :1] - x[:, :1].mean(dim=2, keepdim=True)
        x = torch.cat([x0, x[:, 1:]], dim=1)
        sq = torch.zeros(x.shape[0], L + 1, x.shape[2], device=x.device, dtype=x.dtype)
        sq.index_add_(1, self._deg, x * x)
        if self.normalization == "component":
            sq = sq / (2 * torch.arange(L + 1, device=x.device, dtype=x.dtype) + 1).view(1, -1, 1)
        scale = (sq.mean(dim=2, keepdim=True) + self.eps).rsqrt()  # [N, L+1, 1]
        if self.affine:
            scale = scale * self.affine_weight.unsqueeze(0)
        out = x * scale.index_select(1, self._deg)
        if self.affine:
            out = torch.cat([out[:, :1] + self.affine_bias.view(1, 1, -1), out[:, 1:]], dim=1)
        return out


class EquivariantLayerNormArraySphericalHarmonics(_ResidualNorm):
    """``layer_norm_sh``: a standard LayerNorm on l = 0 (``norm_l0``), and one degree-balanced
    RMS over all components with l > 0 (weights 1 / ((2l+1) L)) scaled by a per-l weight.
    Reference ``helm/nn/layer_norm.py:122-227``."""

    def __init__(self, lmax: int, num_channels: int, eps: float = 1e-5, affine: bool = True,
                 normalization: str = "component", std_balance_degrees: bool = True):
        super().__init__()
        if normalization not in ("norm", "component"):
            raise ValueError(normalization)
        self.lmax, self.num_channels, self.eps, self.affine = lmax, num_channels, eps, affine
        self.normalization, self.std_balance_degrees = normalization, std_balance_degrees
        self.norm_l0 = nn.LayerNorm(num_channels, eps=eps, elementwise_affine=affine)
        if affine:
            self.affine_weight = nn.Parameter(torch.ones(lmax, num_channels))
        else:
            self.register_parameter("affine_weight", None)
        if std_balance_degrees:
            bw = torch.zeros((lmax + 1) ** 2 - 1, 1)
            for l in range(1, lmax + 1):
                bw[l * l - 1: l * l - 1 + 2 * l + 1] = 1.0 / (2 * l + 1)
            self.register_buffer("balance_degree_weight", bw / max(lmax, 1))
        else:
            self.balance_degree_weight = None
        self.register_buffer("_deg", l_expand_index(lmax)[1:] - 1, persistent=False)

    def normalize(self, x):
        out0 = self.norm_l0(x[:, :1])
        if self.lmax == 0:
            return out0
        f = x[:, 1:]
        if self.normalization == "norm":
            n = (f * f).sum(dim=1, keepdim=True)
        elif self.std_balance_degrees:
            n = torch.einsum("nic,ia->nac", f * f, self.balance_degree_weight)
        else:
            n = (f * f).mean(dim=1, keepdim=True)
        scale = (n.mean(dim=2, keepdim=True) + self.eps).rsqrt()  # [N, 1, 1]
        if self.affine:
            scale = scale * self.affine_weight.index_select(0, self._deg).unsqueeze(0)
        return torch.cat([out0, f * scale], dim=1)


class EquivariantDegreeLayerScale(nn.Module):
    """Per-degree layer scale: ``x * affine_weight[l]`` with the l > 0 weights initialised to
    1/sqrt(scale_factor * l).  Reference ``helm/nn/layer_norm.py:341-370``."""

    def __init__(self, lmax: int, num_channels: int, scale_factor: float = 2.0):
        super().__init__()
        self.lmax, self.num_channels, self.scale_factor = lmax, num_channels, scale_factor
        w = torch.ones(1, lmax + 1, num_channels)
        for l in range(1, lmax + 1):
            w[0, l] /= math.sqrt(scale_factor * l)
        self.affine_weight = nn.Parameter(w)
        self.register_buffer("expand_index", l_expand_index(lmax))

    def forward(self, x):
        return x * self.affine_weight.index_select(1, self.expand_index)


NORM_TYPES = ("layer_norm", "layer_norm_sh", "rms_norm_sh")


def get_normalization_layer(norm_type: str, lmax: int, num_channels: int, eps: float = 1e-5):
    """The reference's three equivariant norms by name (``helm/nn/layer_norm.py:18-35``);
    ``rms_norm_sh`` (the default) runs on the fused norm kernel."""
    if norm_type == "rms_norm_sh":
        return EquivariantRMSNorm(lmax, num_channels, eps)
    if norm_type == "layer_norm":
        return EquivariantLayerNormArray(lmax, num_channels, eps)
    if norm_type == "layer_norm_sh":
        return EquivariantLayerNormArraySphericalHarmonics(lmax, num_channels, eps)
    raise ValueError(f"unknown norm_type {norm_type!r}; one of {NORM_TYPES}")


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


class SO2_Linear(nn.Module):
    """SO(2) linear over all |m| <= mmax without the complex pairing: m = 0 is one linear
    over its (l, channel) entries (with bias); for m > 0 the +m and -m rows each go through
    the same bias-free linear.  Inputs and outputs are l-major [E, (L+1)^2, C]; entries with
    |m| > mmax are zero on output.  Optional radial modulation of the inputs from
    ``edge_channels_list``.  Reference ``helm/nn/so2_layers.py:217-328`` (unused by default).
    """

    def __init__(self, sphere_channels, m_output_channels, lmax, mmax, mappingReduced=None, internal_weights=False,
                 edge_channels_list=None):
        super().__init__()
        self.sphere_channels, self.m_output_channels = sphere_channels, m_output_channels
        self.lmax, self.mmax = lmax, mmax
        self.mapping = mappingReduced or CoefficientMapping(lmax, mmax)
        self.internal_weights = internal_weights
        n0 = (lmax + 1) * sphere_channels
        self.fc_m0 = nn.Linear(n0, m_output_channels * (lmax + 1), bias=True)
        n_rad = n0
        self.so2_m_fc = nn.ModuleList()
        for m in range(1, mmax + 1):
            k = (lmax - m + 1) * sphere_channels
            self.so2_m_fc.append(nn.Linear(k, m_output_channels * (lmax - m + 1), bias=False))
            n_rad += k
        self.rad_func = None
        if not internal_weights:
            if edge_channels_list is None:
                raise ValueError("SO2_Linear with radial weights needs edge_channels_list")
            self.rad_func = RadialMLP(list(edge_channels_list) + [int(n_rad)])

    def forward(self, x, x_edge):
        E, C = x.shape[0], self.m_output_channels
        xm = x.index_select(1, self.mapping.m_to_lm)  # m-major
        rad = self.rad_func(x_edge) if self.rad_func is not None else None
        sizes = self.mapping.m_size
        x0 = xm[:, : sizes[0]].reshape(E, -1)
        if rad is not None:
            x0 = x0 * rad[:, : x0.shape[1]]
        outs = [self.fc_m0(x0).view(E, -1, C)]
        off, roff = sizes[0], x0.shape[1]
        for m in range(1, self.mmax + 1):
            k = sizes[m]
            xk = xm[:, off: off + 2 * k].reshape(E, 2, -1)
            if rad is not None:
                xk = xk * rad[:, roff: roff + xk.shape[2]].unsqueeze(1)
                roff += xk.shape[2]
            outs.append(self.so2_m_fc[m - 1](xk).view(E, -1, C))
            off += 2 * k
        out_m = torch.cat(outs, dim=1)
        out = out_m.new_zeros(E, (self.lmax + 1) ** 2, C)
        out[:, self.mapping.m_to_lm] = out_m
        return out


def _fejer_weights(n: int) -> "np.ndarray":
    """Fejer's first quadrature rule on [0, pi] in theta (midpoint nodes (k + 1/2) pi / n):
    sum_k w_k g(cos theta_k) = int_0^pi g(cos theta) sin theta dtheta, exact for polynomials
    in cos(theta) of degree < n."""
    import numpy as np

    th = (np.arange(n) + 0.5) * np.pi / n
    w = np.ones(n)
    for j in range(1, n // 2 + 1):
        w -= 2 * np.cos(2 * j * th) / (4 * j * j - 1)
    return w * 2.0 / n


class SO3_Grid(nn.Module):
    """Matrices between l-major coefficients (|m| <= mmax) and values on an S^2 grid of
    ``lat_resolution`` polar angles (midpoints) x ``long_resolution`` azimuths.

    ``to_grid_mat[b, a, i]`` is the real spherical harmonic i at grid point (b, a) (y polar
    axis); ``from_grid_mat`` is the same harmonic times the quadrature weight (Fejer's first
    rule in the polar angle, uniform in azimuth), so from(to(x)) = x for coefficients up to
    ``lmax``.  ``normalization='integral'`` gives harmonics with unit integral of the square,
    ``'component'`` unit mean.  With mmax < lmax and ``rescale`` the l > mmax rows are scaled by
    sqrt((2l+1)/(2 mmax+1)).  Reference ``helm/common/so3.py:165-264`` (which builds the same
    matrices from e3nn's grids; unused by default).
    """

    def __init__(self, lmax: int, mmax: int, normalization: str = "integral", resolution: int | None = None,
                 rescale: bool = True):
        super().__init__()
        import numpy as np

        from ..core.sph import real_sph_harm

        self.lmax, self.mmax, self.rescale = lmax, mmax, rescale
        self.lat_resolution = 2 * (lmax + 1)
        self.long_resolution = 2 * (mmax + 1) + 1 if lmax == mmax else 2 * mmax + 1
        if resolution is not None:
            self.lat_resolution = self.long_resolution = resolution
        nb, na = self.lat_resolution, self.long_resolution
        beta = (np.arange(nb) + 0.5) * np.pi / nb
        alpha = np.arange(na) * 2 * np.pi / na
        B, A = np.meshgrid(beta, alpha, indexing="ij")
        pts = np.stack([np.sin(B) * np.sin(A), np.cos(B), np.sin(B) * np.cos(A)], -1).reshape(-1, 3)
        Y = np.concatenate([real_sph_harm(l, pts) for l in range(lmax + 1)], 1)  # component norm
        if normalization == "integral":
            Y = Y / math.sqrt(4 * math.pi)
            inv_norm = 1.0
        elif normalization == "component":
            inv_norm = 1.0 / (4 * math.pi)
        else:
            raise ValueError(normalization)
        w = (_fejer_weights(nb)[:, None] * np.full((1, na), 2 * np.pi / na)).reshape(-1, 1)
        to = Y.reshape(nb, na, -1)
        frm = (Y * w * inv_norm).reshape(nb, na, -1)
        ls = np.concatenate([[l] * (2 * l + 1) for l in range(lmax + 1)])
        ms = np.concatenate([np.arange(-l, l + 1) for l in range(lmax + 1)])
        if rescale and lmax != mmax:
            f = np.where(ls > mmax, np.sqrt((2 * ls + 1) / (2 * mmax + 1)), 1.0)
            to, frm = to * f, frm * f
        keep = np.flatnonzero(np.abs(ms) <= mmax)
        self.register_buffer("to_grid_mat", torch.tensor(to[:, :, keep], dtype=torch.float32), persistent=False)
        self.register_buffer("from_grid_mat", torch.tensor(frm[:, :, keep], dtype=torch.float32),
                             persistent=False)

    def get_to_grid_mat(self, device=None):
        return self.to_grid_mat

    def get_from_grid_mat(self, device=None):
        return self.from_grid_mat

    def to_grid(self, embedding, lmax=None, mmax=None):
        return torch.einsum("bai,zic->zbac", self.to_grid_mat.to(embedding.dtype), embedding)

    def from_grid(self, grid, lmax=None, mmax=None):
        return torch.einsum("bai,zbac->zic", self.from_grid_mat.to(grid.dtype), grid)


class S2Activation(nn.Module):
    """SiLU applied pointwise on the S^2 grid: to grid, SiLU, back to coefficients.
    ``SO3_grid`` is an :class:`SO3_Grid` or a dict holding one under ``'lmax_mmax'``
    (the reference's form, ``helm/nn/activation.py:80-96``)."""

    def __init__(self, lmax: int, mmax: int, SO3_grid):
        super().__init__()
        self.lmax, self.mmax = lmax, mmax
        self.SO3_grid = SO3_grid["lmax_mmax"] if isinstance(SO3_grid, (dict, nn.ModuleDict)) else SO3_grid

    def forward(self, inputs):
        return self.SO3_grid.from_grid(torch.nn.functional.silu(self.SO3_grid.to_grid(inputs)))


class SeparableS2Activation(nn.Module):
    """SiLU on the scalars, S^2 activation on the rest; the l = 0 entry of the output is the
    activated scalar (reference ``helm/nn/activation.py:99-120``)."""

    def __init__(self, lmax: int, mmax: int, SO3_grid):
        super().__init__()
        self.lmax, self.mmax = lmax, mmax
        self.s2_act = S2Activation(lmax, mmax, SO3_grid)

    def forward(self, input_scalars, input_tensors):
        s = torch.nn.functional.silu(input_scalars).reshape(input_scalars.shape[0], 1, input_scalars.shape[-1])
        t = self.s2_act(input_tensors)
        return torch.cat([s, t[:, 1:]], dim=1)
